// Device bodies of the forward's row operations (one activation row per
// block): embedding gather, materialised RMSNorm(s), and the final argmax
// over per-block partials of the logits GEMV.  Shared by the standalone
// kernels (rows.cu) and the persistent forward kernel.
#pragma once
#include "act.cuh"
#include "common.cuh"
#include "kernels.cuh"

namespace alm {

constexpr int kRowThreads = 256;

// androidllm/engine.py:280 (embed[token]) with the table dequantized on the
// fly exactly like androidllm/engine.py:98-105: fp16(q * scale) per element.
ALM_DEV void embed_body(const EmbedArgs& a, int m) {
  const int tok = a.tokens[m];
  const bool ok = tok >= 0 && tok < a.vocab;
  if (!ok && threadIdx.x == 0 && a.err) *a.err = 1;
  half* out = a.out + static_cast<size_t>(m) * a.hidden;
  for (int k = threadIdx.x; k < a.hidden; k += kRowThreads) {
    half v = __ushort_as_half(0);
    if (ok) {
      const size_t row = static_cast<size_t>(tok);
      if (a.bits == 16) {
        v = reinterpret_cast<const half*>(a.table)[row * a.row_bytes / 2 + k];
      } else {
        int q;
        const uint8_t* p = static_cast<const uint8_t*>(a.table) + row * a.row_bytes;
        if (a.bits == 8) {
          q = static_cast<int8_t>(p[k]);
        } else {
          const int nib = (k & 1) ? (p[k / 2] >> 4) : (p[k / 2] & 0xf);
          q = nib >= 8 ? nib - 16 : nib;
        }
        v = __hmul(__int2half_rn(q), a.scale[row * a.nsb + k / a.block]);
      }
    }
    out[k] = v;
  }
}

// Fixed-order block sum: per-thread strided sequential sums, then a tree.
ALM_DEV float block_sum(float v, float* red) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fadd(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) red[warp] = v;
  body_sync();
  float s = 0.f;
  for (int w = 0; w < kRowThreads / kWarp; ++w) s = fadd(s, red[w]);
  body_sync();
  return s;
}

struct RowShared {
  float red[kRowThreads / kWarp];
  float den;
  float sv[kRowThreads];
  int si[kRowThreads];
};

// xrow: H halves of shared memory.
ALM_DEV void rownorm_body(const ActIn& in, const half* w2, float eps2, half* out, int ldo, int m, half* xrow,
                          RowShared& sh) {
  float* red = sh.red;
  const int H = in.H;
  if (in.ss && threadIdx.x < kWarp) {
    const float d = row_denominator(in, m);
    if (threadIdx.x == 0) sh.den = d;
  }
  body_sync();
  const float den = in.ss ? sh.den : 1.f;
  float sq = 0.f;
  const int n8 = (H + 7) / 8;
  for (int base = 0; base < n8; base += kRowThreads * 4) {
    uint4 raw[4], wv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = base + j * kRowThreads + threadIdx.x;
      raw[j] = c < n8 ? load_row8(in, m, c * 8, H) : make_uint4(0, 0, 0, 0);
      wv[j] = (c < n8 && in.ss) ? load_w8(in.w, c * 8, H, in.vec) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = base + j * kRowThreads + threadIdx.x;
      if (c >= n8) break;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int k = c * 8 + e;
        if (k >= H) break;
        float v = u4_half(raw[j], e);
        if (in.ss) v = norm_value(v, den, u4_half(wv[j], e));
        xrow[k] = __float2half_rn(v);
        sq = fadd(sq, fmul(v, v));
      }
    }
  }
  body_sync();
  half* o = out + static_cast<size_t>(m) * ldo;
  if (w2 == nullptr) {
    for (int k = threadIdx.x; k < H; k += kRowThreads) o[k] = xrow[k];
  } else {
    const float tot = block_sum(sq, red);
    const float den2 = sqrtf(fadd(fdiv(tot, static_cast<float>(H)), eps2));
    for (int k = threadIdx.x; k < H; k += kRowThreads)
      o[k] = __float2half_rn(fmul(fdiv(__half2float(xrow[k]), den2), __half2float(__ldg(w2 + k))));
  }
  body_sync();   // xrow is reused by the caller's next block
}

// Best (value, index) of row m's per-CTA argmax partials (larger value, then
// smaller index); every thread gets the pair.
ALM_DEV void argmax_reduce_body(const float* am_val, const int* am_idx, int n_part, int m, RowShared& sh,
                                float& best_v, int& best_i) {
  float* sv = sh.sv;
  int* si = sh.si;
  float bv = kNegInf;
  int bi = 0x7fffffff;
  for (int base = 0; base < n_part; base += kRowThreads * 8) {
    float v[8];
    int ix[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + j * kRowThreads + threadIdx.x;
      v[j] = i < n_part ? __ldcg(am_val + static_cast<size_t>(m) * n_part + i) : kNegInf;
      ix[j] = i < n_part ? __ldcg(am_idx + static_cast<size_t>(m) * n_part + i) : 0x7fffffff;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (better(v[j], ix[j], bv, bi)) { bv = v[j]; bi = ix[j]; }
  }
  sv[threadIdx.x] = bv;
  si[threadIdx.x] = bi;
  body_sync();
  for (int s = kRowThreads / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s && better(sv[threadIdx.x + s], si[threadIdx.x + s], sv[threadIdx.x], si[threadIdx.x])) {
      sv[threadIdx.x] = sv[threadIdx.x + s];
      si[threadIdx.x] = si[threadIdx.x + s];
    }
    body_sync();
  }
  best_v = sv[0];
  best_i = si[0];
  body_sync();
}

ALM_DEV void argmax_final_body(const float* am_val, const int* am_idx, int n_part, int* out, int m,
                               RowShared& sh) {
  float bv;
  int bi;
  argmax_reduce_body(am_val, am_idx, n_part, m, sh, bv, bi);
  if (threadIdx.x == 0) out[m] = bi == 0x7fffffff ? 0 : bi;
}

}  // namespace alm
