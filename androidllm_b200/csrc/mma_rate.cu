// Tensor-core instruction rates on this GPU, measured by the library itself
// (bench.py --mma-rate): they decide which MMA each matmul path uses.
//   * mma.sync m16n8k16 (f16 in, f32 accumulate, register operands): cycles
//     per instruction per SM with W warps per SM and C independent
//     accumulator chains per warp;
//   * tcgen05.mma kind::f16, M = 128, K = 16, one issuing thread per SM: ns
//     per instruction for a given N, A from tensor memory (TS) or shared
//     memory (SS), rotating over NA accumulators.
// Operands are constants; only the issue and completion rates are measured.
#include <vector>

#include "../../include/androidllm_b200.h"
#include "tc.cuh"

namespace alm {
namespace {

template <int C>
__global__ void hmma_rate_kernel(int iters, float* sink, unsigned long long* cycles) {
  float acc[C][4];
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[c][j] = 0.f;
  const uint32_t a0 = 0x3c003c00u ^ threadIdx.x, a1 = 0x3c003c00u, a2 = a0 + 1, a3 = a1 + 7;
  const uint32_t b0 = 0x3c00u, b1 = 0x3c01u;
  __syncthreads();
  const unsigned long long t0 = clock64();
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int c = 0; c < C; ++c)
      asm volatile(
          "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
          : "+f"(acc[c][0]), "+f"(acc[c][1]), "+f"(acc[c][2]), "+f"(acc[c][3])
          : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  __syncthreads();
  const unsigned long long t1 = clock64();
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c)
#pragma unroll
    for (int j = 0; j < 4; ++j) s += acc[c][j];
  sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
  if (threadIdx.x == 0) cycles[blockIdx.x] = t1 - t0;
}

// 16 KB of shared memory: A (128 x 16 fp16, K-major core matrices) at 0,
// B (up to 256 x 16) at 4096.  Tensor memory: A in columns 0..7, the
// accumulators from column 256 (na * n <= 256).
__global__ void tc_rate_kernel(int ts, int n, int na, int iters, unsigned long long* ns, int* status) {
  extern __shared__ __align__(1024) unsigned char sm[];
  __shared__ uint32_t tbase;
  __shared__ __align__(8) uint64_t bar;
  const int warp = threadIdx.x / 32;
  for (int i = threadIdx.x; i < 12288 / 2; i += blockDim.x) reinterpret_cast<uint16_t*>(sm)[i] = 0x3c00;
  fence_proxy_async_smem();
  if (warp == 0) tc_alloc(&tbase, 512);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t t = tbase;
  {
    uint32_t r[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) r[c] = 0x3c003c00u;
    tc_st32(tc_addr(t, warp * 32, 0), r);
    tc_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    tc_fence_after();
    const uint32_t idesc = tc_idesc_f16(128, n);
    const uint64_t adesc = tc_sdesc(smem_addr(sm), 128 * 16, 128);
    const uint64_t bdesc = tc_sdesc(smem_addr(sm) + 4096, static_cast<uint32_t>(n) * 16, 128);
    const unsigned long long t0 = global_ns();
    for (int i = 0; i < iters; ++i) {
      const uint32_t d = t + 256 + static_cast<uint32_t>((i % na) * n);
      if (ts) {
        tc_mma_ts(d, t, bdesc, idesc, i >= na);
      } else {
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(i >= na ? 1 : 0)
            : "memory");
      }
    }
    tc_commit(&bar);
    if (!mbar_wait(&bar, 0)) atomicExch(status, 1);
    ns[blockIdx.x] = global_ns() - t0;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_dealloc(t, 512);
  }
}

}  // namespace
}  // namespace alm

int alm_internal_fail(int code, const char* msg);
int alm_internal_ctx(alm_ctx* ctx, int* device, cudaStream_t* stream);

int alm_bench_mma_rate(alm_ctx* ctx, int kind, int n_or_warps, int acc_or_chains, double* result) {
  using namespace alm;
  if (!ctx || !result) return alm_internal_fail(ALM_ERR_ARG, "null argument");
  int device = 0;
  cudaStream_t st = nullptr;
  int rc = alm_internal_ctx(ctx, &device, &st);
  if (rc) return rc;
  int n_sms = 148;
  cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, device);
  void* buf = nullptr;        // mma.sync sink: one float per thread
  int* status = nullptr;
  unsigned long long* dv = nullptr;   // per-CTA cycles or nanoseconds
  if (cudaMalloc(&buf, static_cast<size_t>(n_sms) * 1024 * sizeof(float)) != cudaSuccess ||
      cudaMalloc(&status, sizeof(int)) != cudaSuccess ||
      cudaMalloc(&dv, static_cast<size_t>(n_sms) * sizeof(unsigned long long)) != cudaSuccess) {
    cudaFree(buf);
    cudaFree(status);
    return alm_internal_fail(ALM_ERR_CUDA, "allocation failed");
  }
  cudaMemsetAsync(status, 0, sizeof(int), st);
  std::vector<unsigned long long> h(n_sms);
  cudaError_t e = cudaSuccess;
  if (kind == 0) {
    const int warps = n_or_warps, chains = acc_or_chains, iters = 4096;
    if (warps < 1 || warps > 32 || (chains != 1 && chains != 2 && chains != 4 && chains != 8)) {
      cudaFree(buf);
      cudaFree(status);
      cudaFree(dv);
      return alm_internal_fail(ALM_ERR_ARG, "mma.sync rate: 1..32 warps, 1/2/4/8 chains");
    }
    for (int rep = 0; rep < 2 && e == cudaSuccess; ++rep) {
      float* sink = static_cast<float*>(buf);
      switch (chains) {
        case 1: hmma_rate_kernel<1><<<n_sms, warps * 32, 0, st>>>(iters, sink, dv); break;
        case 2: hmma_rate_kernel<2><<<n_sms, warps * 32, 0, st>>>(iters, sink, dv); break;
        case 4: hmma_rate_kernel<4><<<n_sms, warps * 32, 0, st>>>(iters, sink, dv); break;
        default: hmma_rate_kernel<8><<<n_sms, warps * 32, 0, st>>>(iters, sink, dv); break;
      }
      e = cudaStreamSynchronize(st);
    }
    if (e == cudaSuccess) e = cudaMemcpy(h.data(), dv, n_sms * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    double c = 0;
    for (auto v : h) c += static_cast<double>(v);
    *result = c / n_sms / (static_cast<double>(iters) * chains * warps);   // cycles per MMA per SM
  } else {
    const int n = n_or_warps, na = acc_or_chains, iters = 2048;
    if ((kind != 1 && kind != 2) || n < 16 || n > 256 || n % 16 || na < 1 || na * n > 256) {
      cudaFree(buf);
      cudaFree(status);
      cudaFree(dv);
      return alm_internal_fail(ALM_ERR_ARG, "tcgen05 rate: kind 1 (TS) or 2 (SS), N multiple of 16 in 16..256, acc*N <= 256");
    }
    e = cudaFuncSetAttribute(tc_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 16384);
    for (int rep = 0; rep < 2 && e == cudaSuccess; ++rep) {
      tc_rate_kernel<<<n_sms, 128, 16384, st>>>(kind == 1 ? 1 : 0, n, na, iters, dv, status);
      e = cudaStreamSynchronize(st);
    }
    int hs = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&hs, status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(h.data(), dv, n_sms * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    double t = 0;
    for (auto v : h) t += static_cast<double>(v);
    *result = t / n_sms / iters;   // ns per MMA
    if (e == cudaSuccess && hs) e = cudaErrorTimeout;
  }
  cudaFree(buf);
  cudaFree(status);
  cudaFree(dv);
  if (e != cudaSuccess) return alm_internal_fail(ALM_ERR_CUDA, cudaGetErrorString(e));
  return 0;
}
