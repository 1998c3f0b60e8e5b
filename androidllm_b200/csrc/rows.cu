// Row kernels of the forward: embedding gather, materialised RMSNorm(s) and
// the final argmax over per-CTA partials of the logits GEMV.
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
  grid_dep_wait();
  const int m = blockIdx.x;
  const int H = in.H;
  float den = 1.f;
  if (in.ss) {
    const float* p = in.ss + static_cast<size_t>(m) * in.n_ss;
    float s = 0.f;
    for (int i = 0; i < in.n_ss; ++i) s = fadd(s, p[i]);
    den = sqrtf(fadd(fdiv(s, static_cast<float>(H)), in.eps));
  }
  float sq = 0.f;
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    float v = __half2float(in.x[static_cast<size_t>(m) * in.ld + k]);
    if (in.ss) v = round_h(fmul(fdiv(v, den), __half2float(in.w[k])));
    xrow[k] = __float2half_rn(v);
    sq = fadd(sq, fmul(v, v));
  }
  half* o = out + static_cast<size_t>(m) * ldo;
  if (w2 == nullptr) {
    for (int k = threadIdx.x; k < H; k += blockDim.x) o[k] = xrow[k];
    return;
  }
  const float tot = block_sum(sq, red);
  const float den2 = sqrtf(fadd(fdiv(tot, static_cast<float>(H)), eps2));
  for (int k = threadIdx.x; k < H; k += blockDim.x)
    o[k] = __float2half_rn(fmul(fdiv(__half2float(xrow[k]), den2), __half2float(w2[k])));
}

ALM_DEV bool better(float v1, int i1, float v2, int i2) { return v1 > v2 || (v1 == v2 && i1 < i2); }

__global__ void argmax_final_kernel(const float* am_val, const int* am_idx, int n_part, int* out) {
  __shared__ float sv[kRowThreads];
  __shared__ int si[kRowThreads];
  grid_dep_wait();
  const int m = blockIdx.x;
  float bv = kNegInf;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n_part; i += blockDim.x) {
    const float v = am_val[static_cast<size_t>(m) * n_part + i];
    const int ix = am_idx[static_cast<size_t>(m) * n_part + i];
    if (better(v, ix, bv, bi)) { bv = v; bi = ix; }
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

cudaError_t launch_rownorm(const ActIn& in, int M, const half* w2, float eps2, half* out, int ldo,
                           bool pdl, cudaStream_t st) {
  if (in.H > 24576) return cudaErrorInvalidValue;
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
