// Source access shared by the weight repack kernels (qweight.cu for the
// tile layout, tc_gemv.cu for the row layout).
#pragma once
#include "kernels.cuh"

namespace alm {

struct SrcSet {
  const uint8_t* data[3];
  const half* scale[3];
};

// Signed code (or raw fp16 bits) of source row `row` (src index in the top
// byte of `desc`) at column `col`; zero past the stored columns or for
// padding rows (desc < 0).
__device__ inline int fetch_code(const SrcSet& s, int desc, int col, int bits, int k_pad) {
  if (desc < 0 || col >= k_pad) return 0;
  const int si = desc >> 24;
  const size_t row = static_cast<size_t>(desc & 0xffffff);
  const uint8_t* p = s.data[si];
  if (bits == 4) {
    const uint8_t b = p[row * (k_pad / 2) + col / 2];
    const int nib = (col & 1) ? (b >> 4) : (b & 0xf);
    return nib >= 8 ? nib - 16 : nib;
  }
  if (bits == 8) return static_cast<int8_t>(p[row * k_pad + col]);
  return reinterpret_cast<const uint16_t*>(p)[row * k_pad + col];
}

}  // namespace alm
