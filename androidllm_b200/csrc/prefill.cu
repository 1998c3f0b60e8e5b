// Row kernels of the batched prefill (alm_prefill): the dense tcgen05 path
// stores plain fp16 matmul outputs for up to 256 rows, and these kernels do
// what the M <= 16 path's fused epilogues do, with the same operations:
//   * RoPE on q and k (fp32 on the fp16-rounded projections, the fp16 cos /
//     sin table; androidllm/models/llama.py:42-49,101-104), q kept in fp32
//     for the attention's hi/lo split, k and v stored fp16 into the paged
//     cache (llama.py:105-107);
//   * SwiGLU: fp16(silu(g) * u) in fp32 from the fp16 gate / up outputs
//     (llama.py:52-55,121).
// The residual adds and the norms reuse the row kernels of rows.cu.
#include "common.cuh"
#include "kernels.cuh"

namespace alm {
namespace {

constexpr int kPfThreads = 256;

// One block per row m (position pos0 + m).  Columns of qkv: q heads, k
// heads, v heads (head_dim each).
__global__ void __launch_bounds__(kPfThreads) pf_rope_kv_kernel(PfRopeArgs a) {
  grid_dep_wait();
  const int m = blockIdx.x;
  const int pos = a.pos0 + m;
  const int hd = a.head_dim, half_d = hd / 2;
  const int qd = a.heads * hd, kd = a.kv_heads * hd;
  const half* row = a.qkv + static_cast<size_t>(m) * a.ld_qkv;
  const half* cs = a.rope + static_cast<size_t>(pos) * hd;
  const int page = a.page_table[pos / a.page_size];
  const int slot = pos % a.page_size;
  // RoPE pairs (d, d + head_dim / 2) of the q and k heads
  const int n_pairs = (a.heads + a.kv_heads) * half_d;
  for (int i = threadIdx.x; i < n_pairs; i += kPfThreads) {
    const int head = i / half_d, d = i % half_d;
    const bool is_q = head < a.heads;
    const int col = is_q ? head * hd + d : qd + (head - a.heads) * hd + d;
    const float x0 = __half2float(row[col]), x1 = __half2float(row[col + half_d]);
    const float c = __half2float(__ldg(cs + d)), s = __half2float(__ldg(cs + half_d + d));
    const float rlo = fsub(fmul(x0, c), fmul(x1, s));
    const float rhi = fadd(fmul(x0, s), fmul(x1, c));
    if (is_q) {
      float* q = a.q + static_cast<size_t>(m) * a.ldq + head * hd;
      q[d] = rlo;
      q[d + half_d] = rhi;
    } else {
      const int kh = head - a.heads;
      half* kp = a.kcache + ((static_cast<size_t>(page) * a.kv_heads + kh) * a.page_size + slot) * hd;
      kp[d] = __float2half_rn(rlo);
      kp[d + half_d] = __float2half_rn(rhi);
    }
  }
  for (int i = threadIdx.x; i < kd; i += kPfThreads) {
    const int kh = i / hd, d = i % hd;
    half* vp = a.vcache + ((static_cast<size_t>(page) * a.kv_heads + kh) * a.page_size + slot) * hd;
    vp[d] = row[qd + kd + i];
  }
  grid_dep_launch();
}

// h[m][j] = fp16(g * sigmoid(g) * u), g = gu[m][j], u = gu[m][inter + j].
__global__ void __launch_bounds__(kPfThreads) pf_swiglu_kernel(const half* gu, int ld_gu, int inter, half* h,
                                                               int ld_h) {
  grid_dep_wait();
  const int m = blockIdx.y;
  const half* row = gu + static_cast<size_t>(m) * ld_gu;
  for (int j = blockIdx.x * kPfThreads + threadIdx.x; j < inter; j += gridDim.x * kPfThreads) {
    const float gv = __half2float(row[j]);
    const float uv = __half2float(row[inter + j]);
    const float sig = fdiv(1.f, fadd(1.f, expf(-gv)));
    h[static_cast<size_t>(m) * ld_h + j] = __float2half_rn(fmul(fmul(gv, sig), uv));
  }
  grid_dep_launch();
}

cudaLaunchConfig_t pf_cfg(dim3 grid, bool pdl, cudaStream_t st, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t c = {};
  c.gridDim = grid;
  c.blockDim = dim3(kPfThreads);
  c.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return c;
}

}  // namespace

cudaError_t launch_pf_rope_kv(const PfRopeArgs& a, int M, bool pdl, cudaStream_t st) {
  if (M < 1 || a.head_dim % 2 != 0) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = pf_cfg(dim3(M), pdl, st, attr);
  return cudaLaunchKernelEx(&c, pf_rope_kv_kernel, a);
}

cudaError_t launch_pf_swiglu(const half* gu, int ld_gu, int inter, int M, half* h, int ld_h, bool pdl,
                             cudaStream_t st) {
  if (M < 1 || inter < 1) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  const int gx = (inter + 4 * kPfThreads - 1) / (4 * kPfThreads);
  cudaLaunchConfig_t c = pf_cfg(dim3(gx, M), pdl, st, attr);
  return cudaLaunchKernelEx(&c, pf_swiglu_kernel, gu, ld_gu, inter, h, ld_h);
}

}  // namespace alm
