// Row kernels of the forward: embedding gather, materialised RMSNorm(s) and
// the final argmax over per-CTA partials of the logits GEMV.
#include "act.cuh"
#include "common.cuh"
#include "kernels.cuh"

namespace alm {
namespace {

constexpr int kRowThreads = 256;

// androidllm/engine.py:280 (embed[token]) with the table dequantized on the
// fly exactly like androidllm/engine.py:98-105: fp16(q * scale) per element.
__global__ void embed_kernel(EmbedArgs a) {
  grid_dep_wait();
  const int m = blockIdx.x;
  const int tok = a.tokens[m];
  const bool ok = tok >= 0 && tok < a.vocab;
  if (!ok && threadIdx.x == 0 && a.err) *a.err = 1;
  half* out = a.out + static_cast<size_t>(m) * a.hidden;
  for (int k = threadIdx.x; k < a.hidden; k += blockDim.x) {
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
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x / kWarp); ++w) s = fadd(s, red[w]);
  __syncthreads();
  return s;
}

__global__ void rownorm_kernel(ActIn in, const half* w2, float eps2, half* out, int ldo) {
  extern __shared__ half xrow[];
  __shared__ float red[kRowThreads / kWarp];
  __shared__ float s_den;
  grid_dep_wait();
  const int m = blockIdx.x;
  const int H = in.H;
  if (in.ss && threadIdx.x < kWarp) {
    const float d = row_denominator(in, m);
    if (threadIdx.x == 0) s_den = d;
  }
  __syncthreads();
  const float den = in.ss ? s_den : 1.f;
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
  __syncthreads();
  half* o = out + static_cast<size_t>(m) * ldo;
  if (w2 == nullptr) {
    for (int k = threadIdx.x; k < H; k += blockDim.x) o[k] = xrow[k];
    return;
  }
  const float tot = block_sum(sq, red);
  const float den2 = sqrtf(fadd(fdiv(tot, static_cast<float>(H)), eps2));
  for (int k = threadIdx.x; k < H; k += blockDim.x)
    o[k] = __float2half_rn(fmul(fdiv(__half2float(xrow[k]), den2), __half2float(__ldg(w2 + k))));
}

ALM_DEV bool better(float v1, int i1, float v2, int i2) { return v1 > v2 || (v1 == v2 && i1 < i2); }

__global__ void argmax_final_kernel(const float* am_val, const int* am_idx, int n_part, int* out) {
  __shared__ float sv[kRowThreads];
  __shared__ int si[kRowThreads];
  grid_dep_wait();
  const int m = blockIdx.x;
  float bv = kNegInf;
  int bi = 0x7fffffff;
  for (int base = 0; base < n_part; base += blockDim.x * 8) {
    float v[8];
    int ix[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + j * blockDim.x + threadIdx.x;
      v[j] = i < n_part ? __ldcg(am_val + static_cast<size_t>(m) * n_part + i) : kNegInf;
      ix[j] = i < n_part ? __ldcg(am_idx + static_cast<size_t>(m) * n_part + i) : 0x7fffffff;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (better(v[j], ix[j], bv, bi)) { bv = v[j]; bi = ix[j]; }
  }
  sv[threadIdx.x] = bv;
  si[threadIdx.x] = bi;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s && better(sv[threadIdx.x + s], si[threadIdx.x + s], sv[threadIdx.x], si[threadIdx.x])) {
      sv[threadIdx.x] = sv[threadIdx.x + s];
      si[threadIdx.x] = si[threadIdx.x + s];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) out[m] = si[0] == 0x7fffffff ? 0 : si[0];
}

cudaLaunchConfig_t row_cfg(int M, size_t smem, bool pdl, cudaStream_t st, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(M);
  c.blockDim = dim3(kRowThreads);
  c.dynamicSmemBytes = smem;
  c.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return c;
}

}  // namespace

cudaError_t rows_init_attrs() {
  return cudaFuncSetAttribute(rownorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 24576 * 2);
}

cudaError_t launch_embed(const EmbedArgs& a, bool pdl, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = row_cfg(a.M, 0, pdl, st, attr);
  return cudaLaunchKernelEx(&c, embed_kernel, a);
}

cudaError_t launch_rownorm(const ActIn& in_, int M, const half* w2, float eps2, half* out, int ldo,
                           bool pdl, cudaStream_t st) {
  if (in_.H > 24576) return cudaErrorInvalidValue;
  ActIn in = in_;
  set_vec(in);
  cudaLaunchAttribute attr[1];
  const size_t smem = static_cast<size_t>(in.H) * sizeof(half);
  cudaLaunchConfig_t c = row_cfg(M, smem, pdl, st, attr);
  return cudaLaunchKernelEx(&c, rownorm_kernel, in, w2, eps2, out, ldo);
}

cudaError_t launch_argmax_final(const float* am_val, const int* am_idx, int n_part, int M, int* out,
                                bool pdl, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = row_cfg(M, 0, pdl, st, attr);
  return cudaLaunchKernelEx(&c, argmax_final_kernel, am_val, am_idx, n_part, out);
}

}  // namespace alm
