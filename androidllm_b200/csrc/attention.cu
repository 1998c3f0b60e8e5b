// Standalone launches of the two attention passes (bodies in attn_body.cuh).
#include "attn_body.cuh"

namespace alm {
namespace {

__global__ void __launch_bounds__(kAttnThreads) attn_scores_kernel(AttnArgs a, float inv_sqrt_den) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ AttnShared sh;
  attn_scores_pages(a, blockIdx.x, smem_raw);   // the page table is not written by earlier kernels
  __syncthreads();
  attn_scores_body<false>(a, inv_sqrt_den, blockIdx.x, blockIdx.y, blockIdx.z, gridDim.x, smem_raw, sh, DepWait{});
  grid_dep_launch();
}

// One span: grid (16-dim slice, kv head, row group).
__global__ void __launch_bounds__(kAttnThreads) attn_pv_kernel(AttnArgs a, int n_chunks_max) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ AttnShared sh;
  attn_pv_pages(a, smem_raw);
  __syncthreads();
  attn_pv_body<false, false>(a, n_chunks_max, blockIdx.x, blockIdx.y, blockIdx.z, smem_raw, sh, 0, 1, DepWait{});
}

// Span split (KV capacity above one span): grid (16-dim slice, kv head,
// span x row group) with the blocks of span 0 first.  Span 0 stages its
// page numbers before the wait for the scores pass; a later span's block
// first learns the context length and returns at once when it is not needed.
__global__ void __launch_bounds__(kAttnThreads) attn_pv_split_kernel(AttnArgs a, int n_chunks_max, int n_split) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ AttnShared sh;
  const int n_pg = gridDim.z / n_split;
  const int grp = blockIdx.z % n_pg, sp = blockIdx.z / n_pg;
  if (sp == 0) attn_pv_pages(a, smem_raw, 0, n_split);
  __syncthreads();
  grid_dep_wait();
  if (sp > 0) {
    if (sp * kPvSplit >= *a.pos + a.M) return;
    attn_pv_pages(a, smem_raw, sp, n_split);
    __syncthreads();
  }
  attn_pv_body<false, true>(a, n_chunks_max, blockIdx.x, blockIdx.y, grp, smem_raw, sh, sp, n_split);
}

}  // namespace

cudaError_t attention_init_attrs() {
  cudaError_t e = cudaFuncSetAttribute(attn_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(attn_scores_smem(256)));
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(attn_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(attn_pv_smem()));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(attn_pv_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(attn_pv_smem()));
}

cudaError_t launch_attention_scores(const AttnArgs& a, bool pdl, cudaStream_t st) {
  if (a.head_dim % 16 || a.head_dim > 256 || a.heads % a.kv_heads) return cudaErrorInvalidValue;
  const float den = static_cast<float>(sqrt(static_cast<double>(a.head_dim)));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t c1 = {};
  c1.gridDim = dim3(attn_chunks_max(a), a.kv_heads, attn_row_groups(a));
  c1.blockDim = dim3(kAttnThreads);
  c1.dynamicSmemBytes = attn_scores_smem(a.head_dim);
  c1.stream = st;
  c1.attrs = attr;
  c1.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&c1, attn_scores_kernel, a, den);
  if (e == cudaSuccess) prof_mark(3 /* ALM_OP_ATTN_SCORES */, a.M);
  return e;
}

cudaError_t launch_attention(const AttnArgs& a, bool pdl, cudaStream_t st) {
  const cudaError_t e = launch_attention_scores(a, pdl, st);
  if (e != cudaSuccess) return e;
  const int n_chunks_max = attn_chunks_max(a);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const int n_split = a.pv_part ? attn_pv_spans(a.max_ctx) : 1;
  cudaLaunchConfig_t c2 = {};
  c2.blockDim = dim3(kAttnThreads);
  c2.stream = st;
  c2.attrs = attr;
  c2.numAttrs = pdl ? 1 : 0;
  c2.gridDim = dim3(a.head_dim / 16, a.kv_heads, attn_pv_groups(a) * n_split);
  c2.dynamicSmemBytes = attn_pv_smem();
  if (n_split == 1) return cudaLaunchKernelEx(&c2, attn_pv_kernel, a, n_chunks_max);
  return cudaLaunchKernelEx(&c2, attn_pv_split_kernel, a, n_chunks_max, n_split);
}

}  // namespace alm
