// Activation-row helpers shared by the GEMV and the row kernels.
//
// Deferred RMSNorm: a residual-producing GEMV writes the un-normalised row v
// and, per 16-column tile, the fp32 sum of squares of its fp16 values.  A
// consumer rebuilds the RMSNorm denominator from those partials with
// row_denominator() (one warp, fixed order: lane l adds partials l, l+32, ...
// sequentially, then a butterfly), so every kernel that normalises a row gets
// bit-identical values and the result does not depend on how many rows a pass
// carries.  Element: fp16((f32(v) / sqrt(mean + eps)) * f32(w)), the order of
// androidllm/models/llama.py:21-24.
#pragma once
#include "common.cuh"
#include "kernels.cuh"

namespace alm {

// Sum of n fp32 partials, called by all 32 lanes of a warp.
ALM_DEV float warp_fixed_sum(const float* p, int n) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
  for (int base = 0; base < n; base += 32 * 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + j * 32 + lane;
      v[j] = i < n ? __ldcg(p + i) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) s = fadd(s, v[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s = fadd(s, __shfl_xor_sync(0xffffffffu, s, o));
  return s;
}

// sqrt(mean of squares + eps) of row m of a deferred-norm activation.
ALM_DEV float row_denominator(const ActIn& a, int m) {
  const float s = warp_fixed_sum(a.ss + static_cast<size_t>(m) * a.n_ss, a.n_ss);
  return sqrtf(fadd(fdiv(s, static_cast<float>(a.H)), a.eps));
}

// Apply the deferred norm to one raw fp16 value (as fp32) at column k.
ALM_DEV float norm_value(float v, float den, float w) { return round_h(fmul(fdiv(v, den), w)); }

// 8 consecutive raw fp16 values of row m starting at col0 (bounds-checked
// against k_real), packed in a uint4.  Vector load when aligned.
ALM_DEV uint4 load_row8(const ActIn& a, int m, int col0, int k_real) {
  const half* row = a.x + static_cast<size_t>(m) * a.ld;
  if (a.vec && col0 + 8 <= k_real) return __ldcg(reinterpret_cast<const uint4*>(row + col0));
  unsigned short e[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    e[j] = col0 + j < k_real ? __ldcg(reinterpret_cast<const unsigned short*>(row) + col0 + j) : 0;
  return make_uint4(e[0] | (e[1] << 16), e[2] | (e[3] << 16), e[4] | (e[5] << 16), e[6] | (e[7] << 16));
}

// 8 consecutive fp16 norm weights from col0 (zero past k_real).
ALM_DEV uint4 load_w8(const half* w, int col0, int k_real, bool vec) {
  if (vec && col0 + 8 <= k_real) return __ldg(reinterpret_cast<const uint4*>(w + col0));
  unsigned short e[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) e[j] = col0 + j < k_real ? __ldg(reinterpret_cast<const unsigned short*>(w) + col0 + j) : 0;
  return make_uint4(e[0] | (e[1] << 16), e[2] | (e[3] << 16), e[4] | (e[5] << 16), e[6] | (e[7] << 16));
}

ALM_DEV float u4_half(const uint4& v, int j) {
  const uint32_t w = j < 2 ? v.x : j < 4 ? v.y : j < 6 ? v.z : v.w;
  return __half2float(__ushort_as_half(static_cast<unsigned short>((j & 1) ? (w >> 16) : (w & 0xffff))));
}

}  // namespace alm
