// Device-side decoding of the qtile weight layout (see kernels.cuh).
//
// One lane's data for one (tile, k64 block) decodes into the m16n8k16 A
// fragments of four k16 steps.  Codes become exact fp16 integers with the
// 0x6400 exponent trick (1024 + u, then subtract the offset), and the block
// scale is applied with one fp16 multiply, which rounds the exact product
// q * scale to nearest-even: bit-identical to androidllm's
// fp16(f32(q) * f32(scale)) (androidllm/quant.py:58-65).
#pragma once
#include "common.cuh"
#include "kernels.cuh"

namespace alm {

template <int BITS>
struct QTileTraits;
template <>
struct QTileTraits<4> { static constexpr int kVec = 1; };   // uint4 per lane per k64
template <>
struct QTileTraits<8> { static constexpr int kVec = 2; };
template <>
struct QTileTraits<16> { static constexpr int kVec = 4; };

// Record of (tile, kb); codes of vector v of `lane` at rec + v * 32 + lane,
// scale words at reinterpret_cast<const uint32_t*>(rec + kVec * 32) + set * 8 + g.
ALM_DEV const uint4* qtile_record(const QTile& w, int tile, int kb) {
  return w.data + (static_cast<size_t>(tile) * w.k_blocks + kb) * w.rec_u4;
}

// Decode k16 step s of a lane's k64 data into A registers (row g: a0, a2;
// row g+8: a1, a3), scaled by sg (row g) and sg8 (row g+8) for int4/int8.
template <int BITS>
ALM_DEV void decode_step(const uint4 (&wd)[QTileTraits<BITS>::kVec], int s, half2 sg, half2 sg8,
                         uint32_t& a0, uint32_t& a1, uint32_t& a2, uint32_t& a3) {
  if constexpr (BITS == 4) {
    const uint32_t w = s == 0 ? wd[0].x : s == 1 ? wd[0].y : s == 2 ? wd[0].z : wd[0].w;
    const uint32_t w8 = w >> 8;
    const half2 lo = u2h(and_or(w, 0x000f000fu, 0x64006400u));
    const half2 hi = u2h(and_or(w, 0x00f000f0u, 0x64006400u));
    const half2 lo2 = u2h(and_or(w8, 0x000f000fu, 0x64006400u));
    const half2 hi2 = u2h(and_or(w8, 0x00f000f0u, 0x64006400u));
    const half2 off = u2h(0x64086408u);                 // 1032 = 1024 + 8
    const half2 sixteenth = u2h(0x2c002c00u);           // 1/16
    const half2 off16 = u2h(0xd480d480u);               // -72 = -(64 + 8)
    a0 = h2u(__hmul2(__hsub2(lo, off), sg));
    a1 = h2u(__hmul2(__hfma2(hi, sixteenth, off16), sg8));
    a2 = h2u(__hmul2(__hsub2(lo2, off), sg));
    a3 = h2u(__hmul2(__hfma2(hi2, sixteenth, off16), sg8));
  } else if constexpr (BITS == 8) {
    const uint4& v = wd[s >> 1];
    const uint32_t wg = (s & 1) ? v.z : v.x;
    const uint32_t wg8 = (s & 1) ? v.w : v.y;
    const half2 off = u2h(0x64806480u);                 // 1152 = 1024 + 128
    a0 = h2u(__hmul2(__hsub2(u2h(prmt(wg, 0x64646464u, 0x4140u)), off), sg));
    a2 = h2u(__hmul2(__hsub2(u2h(prmt(wg, 0x64646464u, 0x4342u)), off), sg));
    a1 = h2u(__hmul2(__hsub2(u2h(prmt(wg8, 0x64646464u, 0x4140u)), off), sg8));
    a3 = h2u(__hmul2(__hsub2(u2h(prmt(wg8, 0x64646464u, 0x4342u)), off), sg8));
  } else {
    const uint4& v = wd[s];
    a0 = v.x;
    a1 = v.y;
    a2 = v.z;
    a3 = v.w;
  }
}

}  // namespace alm
