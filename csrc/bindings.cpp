// Python bindings of the kvserve_b200 sm_100a extension.  Every op runs on
// the caller's current CUDA stream and does no host synchronisation, so the
// ops can be captured in CUDA graphs.
#include <torch/extension.h>

#include "ops.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "kvserve_b200 sm_100a kernels";
  // fused KV transfer codec
  m.def("kv_frame_geom", &kvs::kv_frame_geom);
  m.def("kv_encode_layer", &kvs::kv_encode_layer);
  m.def("kv_signed_hadamard", &kvs::kv_signed_hadamard);
  m.def("kv_decode_layers", &kvs::kv_decode_layers);
  // modular pipeline kernels
  m.def("bitpack_encode", &kvs::bitpack_encode);
  m.def("bitpack_decode", &kvs::bitpack_decode);
  m.def("codebook_quantize", &kvs::codebook_quantize);
  m.def("codebook_dequantize", &kvs::codebook_dequantize);
  m.def("fwht_rows", &kvs::fwht_rows);
  // lossless codec
  m.def("rze_max_encoded_bytes", &kvs::rze_max_encoded_bytes);
  m.def("rze_scratch_bytes", &kvs::rze_scratch_bytes);
  m.def("rze_encode", &kvs::rze_encode);
  m.def("rze_decode", &kvs::rze_decode);
  // peer memory
  m.def("dev_alloc", &kvs::dev_alloc);
  m.def("dev_free", &kvs::dev_free);
  m.def("ipc_get_handle", [](int64_t p) { return pybind11::bytes(kvs::ipc_get_handle(p)); });
  m.def("ipc_open_handle", [](pybind11::bytes b) { return kvs::ipc_open_handle(std::string(b)); });
  m.def("ipc_close", &kvs::ipc_close);
  m.def("can_access_peer", &kvs::can_access_peer);
  m.def("tensor_from_ptr", &kvs::tensor_from_ptr);
  m.def("fill_u32", &kvs::fill_u32);
  m.def("read_u32", &kvs::read_u32);
  m.def("store_release_u32", &kvs::store_release_u32);
  m.def("publish_token", &kvs::publish_token);
  m.def("take_token", &kvs::take_token);
  m.def("wait_flag", &kvs::wait_flag);
  // engine
  m.def("rmsnorm", &kvs::rmsnorm);
  m.def("rope_qkv", &kvs::rope_qkv);
  m.def("silu_mul", &kvs::silu_mul);
  m.def("embedding", &kvs::embedding);
  m.def("argmax_rows", &kvs::argmax_rows);
  m.def("decode_advance", &kvs::decode_advance);
  m.def("batch_advance", &kvs::batch_advance);
  m.def("gemm_bf16", &kvs::gemm_bf16);
  m.def("gemm_silu_bf16", &kvs::gemm_silu_bf16);
  m.def("gemm_allreduce_bf16", &kvs::gemm_allreduce_bf16);
  m.def("gemm_qkv_rope_bf16", &kvs::gemm_qkv_rope_bf16);
  m.def("gemv_bf16", &kvs::gemv_bf16);
  m.def("gemv_allreduce_bf16", &kvs::gemv_allreduce_bf16);
  m.def("gemv_argmax_bf16", &kvs::gemv_argmax_bf16);
  m.def("decode_epoch_bump", &kvs::decode_epoch_bump);
  m.def("flash_prefill", &kvs::flash_prefill);
  m.def("paged_decode_splits", &kvs::paged_decode_splits);
  m.def("paged_decode_attention", &kvs::paged_decode_attention);
}
