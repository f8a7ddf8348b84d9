// Geometry of one compressed KV "layer frame" — the unit that the prefill
// GPU pushes into the decode GPU's receive slot over NVLink.
//
// A frame holds both parts (K and V) of one layer for one request (one TP
// shard).  Heads are split into two precision sections: section 0 (the
// "low" heads, first in section order) and section 1 (the "high" heads).
// This mirrors the mixed-precision split of the reference quantizer
// (kvserve_v1/compression/quantizer/kvserve_quantizer.py:171-233, low heads
// concatenated first), but the byte layout is this project's own:
//
//   [0, 64)            FrameHeader
//   k_aux              K per-channel  min[H*D] bf16, scale[H*D] bf16
//                      (channels in section-ordered head order)
//   v_aux[s]           V per-token    min[T] bf16, scale[T] bf16, for section s
//   payload[p][s]      one BitPack block per (part, section): the 16-byte
//                      BitPack header (magic 0x0150424B LE, bits, 0,0,0,
//                      count u64 LE) followed by the symbols of shape
//                      [T, heads_in_section, D] packed LSB-first — the exact
//                      format of the reference BitPackCodec
//                      (kvserve_v1/compression/codec/bitpack_codec.py:20-48),
//                      so every section is a self-describing BitPack payload.
//   bits == 16 marks a raw (uncompressed bf16) section: no header, no aux.
//
// Every region starts on a 256-byte boundary.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define KVS_HD __host__ __device__
#else
#define KVS_HD
#endif

namespace kvs {

constexpr uint32_t kFrameMagic = 0x4653564Bu;     // "KVSF"
constexpr uint32_t kBitpackMagic = 0x0150424Bu;   // BitPack format v1
constexpr int kFrameAlign = 256;
constexpr int kRawBits = 16;

struct FrameHeader {
  uint32_t magic;
  uint32_t version;
  uint32_t layer;
  uint32_t tokens;
  uint32_t heads;
  uint32_t head_dim;
  uint32_t n_low;
  uint32_t seq;
  uint8_t bits[2][2];
  uint8_t levels[2][2];
  uint32_t transform;
  uint32_t reserved[5];
};
static_assert(sizeof(FrameHeader) == 64, "frame header is 64 bytes");

struct FrameGeom {
  int32_t T;
  int32_t H;
  int32_t D;
  int32_t n_low;           // heads in section 0
  int32_t bits[2][2];      // [part][section]; 16 = raw bf16
  int32_t levels[2][2];    // quantisation levels (symbols 0..levels-1)
  int32_t transform;       // 1: random-sign Hadamard before quantisation, 0: none
  int64_t k_aux;           // offset of K min/scale
  int64_t v_aux[2];        // offset of V min/scale per section
  int64_t payload[2][2];   // offset of the BitPack block per [part][section]
  int64_t frame_bytes;     // total, multiple of kFrameAlign
};

KVS_HD inline int64_t align_up(int64_t x, int64_t a) {
  return (x + a - 1) / a * a;
}

KVS_HD inline int section_heads(const FrameGeom& g, int s) {
  return s == 0 ? g.n_low : g.H - g.n_low;
}

// Bytes of the packed symbol stream of one (part, section) (excl. header).
KVS_HD inline int64_t section_packed_bytes(const FrameGeom& g, int p, int s) {
  const int64_t count = static_cast<int64_t>(g.T) * section_heads(g, s) * g.D;
  const int b = g.bits[p][s];
  if (b == kRawBits) return count * 2;
  return (count * b + 7) / 8;
}

KVS_HD inline bool section_is_raw(const FrameGeom& g, int p, int s) {
  return g.bits[p][s] == kRawBits;
}

// Fills every offset of `g` from T/H/D/n_low/bits/levels.
// (Written without loops so device code keeps a FrameGeom in registers.)
KVS_HD inline void frame_geom_finalize(FrameGeom& g) {
  int64_t off = align_up(int64_t(sizeof(FrameHeader)), kFrameAlign);
  const bool k_quant = (section_heads(g, 0) > 0 && !section_is_raw(g, 0, 0)) ||
                       (section_heads(g, 1) > 0 && !section_is_raw(g, 0, 1));
  g.k_aux = off;
  if (k_quant) off = align_up(off + 2LL * 2 * g.H * g.D, kFrameAlign);
  g.v_aux[0] = off;
  if (section_heads(g, 0) > 0 && !section_is_raw(g, 1, 0)) off = align_up(off + 2LL * 2 * g.T, kFrameAlign);
  g.v_aux[1] = off;
  if (section_heads(g, 1) > 0 && !section_is_raw(g, 1, 1)) off = align_up(off + 2LL * 2 * g.T, kFrameAlign);
  auto place = [&](int p, int s) -> int64_t {
    const int64_t at = off;
    if (section_heads(g, s) > 0)
      off = align_up(off + (section_is_raw(g, p, s) ? 0 : 16) + section_packed_bytes(g, p, s), kFrameAlign);
    return at;
  };
  g.payload[0][0] = place(0, 0);
  g.payload[0][1] = place(0, 1);
  g.payload[1][0] = place(1, 0);
  g.payload[1][1] = place(1, 1);
  g.frame_bytes = off;
}

}  // namespace kvs
