// Host entry points of the kvserve_b200 CUDA extension (bound in bindings.cpp).
#pragma once
#include <torch/extension.h>

#include <string>
#include <vector>

namespace kvs {

// ---- fused KV transfer codec (kv_codec.cu)
std::vector<int64_t> kv_frame_geom(std::vector<int64_t> params);
// Signed Hadamard table [heads*128, 128] bf16 (rows h*128+o: H[o][i] * sign_h[i]).
torch::Tensor kv_signed_hadamard(torch::Tensor sign_bits);
void kv_encode_layer(torch::Tensor k, torch::Tensor v, std::vector<int64_t> geom, torch::Tensor order,
                     torch::Tensor sign_bits, int64_t frame_ptr, torch::Tensor stats, torch::Tensor counter,
                     int64_t flag_ptr, int64_t seq, int64_t layer, c10::optional<torch::Tensor> pacing,
                     double rate_bytes_per_ns, int64_t max_ctas, int64_t tile_tokens, int64_t part_mask,
                     c10::optional<torch::Tensor> block_table, bool hnd, bool allow_mma,
                     c10::optional<torch::Tensor> hs_table, int64_t hs_row0, int64_t trace_ptr);
void kv_decode_layers(int64_t frame_base, int64_t frame_stride, std::vector<int64_t> geom, torch::Tensor orders,
                      torch::Tensor sign_bits, torch::Tensor kv_cache, torch::Tensor block_table,
                      int64_t tok_offset, int64_t flags_ptr, int64_t seq, int64_t layer_begin, int64_t num_layers,
                      int64_t timeout_ns, torch::Tensor status, int64_t max_ctas, int64_t tile_tokens,
                      c10::optional<torch::Tensor> n_lows, int64_t part_mask,
                      c10::optional<torch::Tensor> layer_ptrs, bool hnd, int64_t trace_ptr);

// ---- modular pipeline kernels (bitpack.cu)
void bitpack_encode(torch::Tensor src, torch::Tensor out, int64_t bits, torch::Tensor status);
void bitpack_decode(torch::Tensor src, torch::Tensor out, int64_t bits, torch::Tensor status);
// ---- centred Gaussian codebook quantiser (codebook.cu); part 0 keys, 1 values
void codebook_quantize(torch::Tensor x, int64_t part, int64_t group, int64_t refinements, double alpha,
                       torch::Tensor centers, torch::Tensor q, torch::Tensor mean, torch::Tensor scale);
void codebook_dequantize(torch::Tensor q, int64_t part, int64_t group, torch::Tensor centers, torch::Tensor mean,
                         torch::Tensor scale, torch::Tensor out, torch::Tensor status);
void fwht_rows(torch::Tensor x, torch::Tensor y, c10::optional<torch::Tensor> signs, bool inverse);

// ---- lossless codec (lossless.cu)
int64_t rze_max_encoded_bytes(int64_t n, int64_t chunk);
int64_t rze_scratch_bytes(int64_t n, int64_t chunk);
void rze_encode(torch::Tensor src, torch::Tensor out, torch::Tensor scratch, torch::Tensor out_total, int64_t chunk);
void rze_decode(torch::Tensor src, torch::Tensor out, torch::Tensor scratch, int64_t chunk);

// ---- peer memory (p2p.cu)
int64_t dev_alloc(int64_t bytes);
void dev_free(int64_t ptr);
std::string ipc_get_handle(int64_t ptr);
int64_t ipc_open_handle(const std::string& handle);
void ipc_close(int64_t ptr);
bool can_access_peer(int64_t dev, int64_t peer);
torch::Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> shape, int64_t dtype_code, int64_t device);
void fill_u32(int64_t ptr, int64_t value, int64_t count);
void read_u32(int64_t ptr, torch::Tensor out);
void store_release_u32(int64_t ptr, int64_t value);
void publish_token(torch::Tensor tok, int64_t dst_ptr, int64_t seq);
void take_token(int64_t src_ptr, int64_t seq, int64_t timeout_ns, torch::Tensor out,
                c10::optional<torch::Tensor> out2, torch::Tensor status);
void wait_flag(int64_t flag_ptr, int64_t target, int64_t timeout_ns, torch::Tensor status);

// ---- engine (engine_ops.cu, gemm_sm100.cu, gemv.cu, attention_*.cu)
void rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor w, torch::Tensor out,
             double eps);
void rope_qkv(torch::Tensor qkv, int64_t Hq, int64_t Hkv, int64_t D, torch::Tensor positions,
              torch::Tensor cos_sin, c10::optional<torch::Tensor> k_dst, c10::optional<torch::Tensor> v_dst,
              int64_t dst_token_stride, int64_t dst_head_stride, c10::optional<torch::Tensor> slot_mapping,
              int64_t slot_base);
void silu_mul(torch::Tensor gate_up, torch::Tensor out, int64_t blk);
void embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out, int64_t vocab_begin);
void argmax_rows(torch::Tensor logits, torch::Tensor out, c10::optional<torch::Tensor> out_val,
                 int64_t index_offset);
void batch_advance(torch::Tensor tok, torch::Tensor active, torch::Tensor ids, torch::Tensor pos, torch::Tensor ctx,
                   torch::Tensor slot, torch::Tensor table, int64_t block_size, torch::Tensor out_tokens,
                   torch::Tensor steps);
void decode_advance(torch::Tensor tok, torch::Tensor ids, torch::Tensor pos, torch::Tensor ctx, torch::Tensor slot,
                    torch::Tensor table, int64_t block_size, torch::Tensor out_tokens, torch::Tensor step);
void gemm_silu_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor err);
// C = all-reduce over tensor-parallel ranks of A_r B_r^T, GEMM and peer-memory
// reduction in one launch (pointers: every rank's C, staging, flags).
void gemm_allreduce_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor c, std::vector<int64_t> out_ptrs,
                         std::vector<int64_t> stage_ptrs, std::vector<int64_t> flag_ptrs, int64_t rank,
                         int64_t max_tiles, int64_t epoch, int64_t timeout_ns, torch::Tensor err);
void gemm_qkv_rope_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor c, c10::optional<torch::Tensor> bias,
                        torch::Tensor cos_sin, torch::Tensor positions, int64_t hq, int64_t hkv,
                        c10::optional<torch::Tensor> k_dst, c10::optional<torch::Tensor> v_dst, torch::Tensor err);
void gemm_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor c, c10::optional<torch::Tensor> residual,
               c10::optional<torch::Tensor> bias, torch::Tensor err);
void gemv_bf16(torch::Tensor x, torch::Tensor w, torch::Tensor y, c10::optional<torch::Tensor> bias);
// decode-step fusions (decode_fused.cu): row-parallel GEMV + one-shot peer
// all-reduce, LM-head GEMV + greedy argmax (+ TP exchange), step epoch
void gemv_allreduce_bf16(torch::Tensor x, torch::Tensor w, torch::Tensor y, std::vector<int64_t> stage_ptrs,
                         int64_t rank, int64_t site, int64_t num_sites, torch::Tensor epoch, int64_t stage_ld,
                         int64_t timeout_ns, torch::Tensor status);
void gemv_argmax_bf16(torch::Tensor x, torch::Tensor w, torch::Tensor out, torch::Tensor part_val,
                      torch::Tensor part_idx, torch::Tensor counter, int64_t vocab_begin,
                      std::vector<int64_t> slot_ptrs, int64_t rank, int64_t site,
                      int64_t num_sites, torch::Tensor epoch, int64_t timeout_ns, torch::Tensor status);
void decode_epoch_bump(torch::Tensor epoch);
void flash_prefill(torch::Tensor qkv, int64_t Hq, int64_t Hkv, double scale, torch::Tensor out, torch::Tensor err,
                   int64_t kstages, int64_t poly);
int64_t paged_decode_splits(int64_t batch, int64_t hkv, int64_t max_ctx);
void paged_decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                            torch::Tensor block_tables, torch::Tensor ctx_lens, int64_t max_ctx, double scale,
                            torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml, int64_t splits);

}  // namespace kvs
