// Row kernels of the forward: embedding gather, materialised RMSNorm(s) and
// the final argmax over per-CTA partials of the logits GEMV (bodies in
// rows_body.cuh).
#include "rows_body.cuh"

namespace alm {
namespace {

__global__ void __launch_bounds__(kRowThreads) embed_kernel(EmbedArgs a) {
  grid_dep_wait();
  embed_body(a, blockIdx.x);
}

__global__ void __launch_bounds__(kRowThreads) rownorm_kernel(ActIn in, const half* w2, float eps2, half* out,
                                                              int ldo) {
  extern __shared__ __align__(16) half xrow[];
  __shared__ RowShared sh;
  grid_dep_wait();
  rownorm_body(in, w2, eps2, out, ldo, blockIdx.x, xrow, sh);
}

__global__ void __launch_bounds__(kRowThreads) argmax_final_kernel(const float* am_val, const int* am_idx,
                                                                   int n_part, int* out) {
  __shared__ RowShared sh;
  grid_dep_wait();
  argmax_final_body(am_val, am_idx, n_part, out, blockIdx.x, sh);
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
