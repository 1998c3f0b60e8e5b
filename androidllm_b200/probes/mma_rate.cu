// Measurement probes, built as a separate library (libalm_probes.so) that
// the product library does not contain or export; `bench.py --mma-rate`
// loads it.  Tensor-core instruction rates on this GPU decide which MMA each
// matmul path uses:
//   * mma.sync m16n8k16 (f16 in, f32 accumulate, register operands): cycles
//     per instruction per SM with W warps per SM and C independent
//     accumulator chains per warp;
//   * tcgen05.mma kind::f16, M = 128, K = 16, one issuing thread per CTA and
//     one or two CTAs per SM: ns per instruction per CTA for a given N, A from
//     tensor memory (TS) or shared memory (SS), rotating over NA accumulators.
// Operands are constants; only the issue and completion rates are measured.
#include <vector>

#include <string>

#include "../csrc/tc.cuh"

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
// B (up to 256 x 16) at 4096.  Tensor memory: `cols` columns (512 / ctas
// per SM), A in columns 0..7, issuer i's `na` accumulators of n columns from
// column 32 + i * na * n.  Issuer i is lane 0 of warp i.
__global__ void tc_rate_kernel(int ts, int n, int na, int iters, int cols, int issuers, unsigned long long* ns,
                               int* status) {
  extern __shared__ __align__(1024) unsigned char sm[];
  __shared__ uint32_t tbase;
  __shared__ __align__(8) uint64_t bar[4];
  const int warp = threadIdx.x / 32;
  for (int i = threadIdx.x; i < 12288 / 2; i += blockDim.x) reinterpret_cast<uint16_t*>(sm)[i] = 0x3c00;
  fence_proxy_async_smem();
  if (warp == 0) tc_alloc(&tbase, cols);
  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&bar[i], 1);
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
    if (warp < 4) tc_st32(tc_addr(t, warp * 32, 0), r);   // columns 0..31: A
    tc_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  if (warp < issuers && (threadIdx.x & 31) == 0) {
    tc_fence_after();
    const uint32_t idesc = tc_idesc_f16(128, n);
    const uint64_t adesc = tc_sdesc(smem_addr(sm), 128 * 16, 128);
    const uint64_t bdesc = tc_sdesc(smem_addr(sm) + 4096, static_cast<uint32_t>(n) * 16, 128);
    const uint32_t d0 = t + 32 + static_cast<uint32_t>(warp * na * n);
    const unsigned long long t0 = global_ns();
    for (int i = 0; i < iters; ++i) {
      const uint32_t d = d0 + static_cast<uint32_t>((i % na) * n);
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
    tc_commit(&bar[warp]);
    if (!mbar_wait(&bar[warp], 0)) atomicExch(status, 1);
    ns[blockIdx.x * issuers + warp] = global_ns() - t0;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_dealloc(t, cols);
  }
}

// An empty dependent kernel: wait for the previous grid, touch one word, let
// the next grid start.  A chain of these measures the per-launch floor of a
// CUDA graph with programmatic dependent launch.
__global__ void nop_chain_kernel(unsigned* word) {
  grid_dep_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) *word += 1;
  grid_dep_launch();
}

}  // namespace
}  // namespace alm

namespace {
thread_local std::string g_probe_err;
int probe_fail(const char* msg) {
  g_probe_err = msg;
  return 1;
}
// A stream on `device` for one probe call.
struct ProbeStream {
  cudaStream_t st = nullptr;
  int n_sms = 148;
  cudaError_t e = cudaSuccess;
  explicit ProbeStream(int device) {
    e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, device);
  }
  ~ProbeStream() {
    if (st) cudaStreamDestroy(st);
  }
};
// ns per tcgen05.mma of each issuing thread; 0 or an ALM error code.
int tc_rate(cudaStream_t st, int n_sms, int ts, int n, int na, int ctas_per_sm, int issuers, double* result) {
  using namespace alm;
  const int cols = 512 / ctas_per_sm, iters = 2048;
  if ((ctas_per_sm != 1 && ctas_per_sm != 2 && ctas_per_sm != 4) || issuers < 1 || issuers > 4 || n < 16 ||
      n > 256 || n % 16 || na < 1 || issuers * na * n > cols - 32)
    return probe_fail(
        "tcgen05 rate: N multiple of 16 in 16..256, 1/2/4 CTAs per SM, 1..4 issuers, "
                             "issuers * accumulators * N <= 512 / ctas_per_sm - 32");
  const size_t n_rec = static_cast<size_t>(ctas_per_sm) * n_sms * issuers;
  int* status = nullptr;
  unsigned long long* dv = nullptr;
  if (cudaMalloc(&status, sizeof(int)) != cudaSuccess ||
      cudaMalloc(&dv, n_rec * sizeof(unsigned long long)) != cudaSuccess) {
    cudaFree(status);
    return probe_fail("allocation failed");
  }
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), st);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(tc_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 16384);
  for (int rep = 0; rep < 2 && e == cudaSuccess; ++rep) {
    tc_rate_kernel<<<ctas_per_sm * n_sms, 128, 16384, st>>>(ts, n, na, iters, cols, issuers, dv, status);
    e = cudaStreamSynchronize(st);
  }
  std::vector<unsigned long long> h(n_rec);
  int hs = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&hs, status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(h.data(), dv, n_rec * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  double t = 0;
  for (auto v : h) t += static_cast<double>(v);
  *result = t / static_cast<double>(n_rec) / iters;
  if (e == cudaSuccess && hs) e = cudaErrorTimeout;
  cudaFree(status);
  cudaFree(dv);
  if (e != cudaSuccess) return probe_fail(cudaGetErrorString(e));
  return 0;
}
}  // namespace

#define PROBE_API extern "C" __attribute__((visibility("default")))

PROBE_API const char* probe_last_error(void) { return g_probe_err.c_str(); }

// tcgen05.mma kind::f16 (M = 128, K = 16) issue rate: ctas_per_sm CTAs on
// every SM, each with `issuers` issuing threads rotating over `accumulators`
// accumulators of N = n columns (A from tensor memory if ts, else shared
// memory).  *ns_per_mma = ns per instruction of one issuing thread.
PROBE_API int probe_tc_rate(int device, int ts, int n, int accumulators, int ctas_per_sm, int issuers,
                            double* ns_per_mma) {
  if (!ns_per_mma) return probe_fail("null argument");
  ProbeStream ps(device);
  if (ps.e != cudaSuccess) return probe_fail(cudaGetErrorString(ps.e));
  return tc_rate(ps.st, ps.n_sms, ts ? 1 : 0, n, accumulators, ctas_per_sm, issuers, ns_per_mma);
}

// kind 0: mma.sync m16n8k16 with n_or_warps warps per SM and acc_or_chains
// (1, 2, 4, 8) accumulator chains per warp, *result = cycles per instruction
// per SM.  kind 1 / 2: tcgen05.mma, A from tensor memory / shared memory, N =
// n_or_warps, rotating over acc_or_chains accumulators, one CTA per SM,
// *result = ns per instruction.
PROBE_API int probe_mma_rate(int device, int kind, int n_or_warps, int acc_or_chains, double* result) {
  using namespace alm;
  if (!result) return probe_fail("null argument");
  ProbeStream ps(device);
  if (ps.e != cudaSuccess) return probe_fail(cudaGetErrorString(ps.e));
  cudaStream_t st = ps.st;
  const int n_sms = ps.n_sms;
  if (kind == 1 || kind == 2) return tc_rate(st, n_sms, kind == 1 ? 1 : 0, n_or_warps, acc_or_chains, 1, 1, result);
  if (kind != 0) return probe_fail("kind 0 (mma.sync), 1 (tcgen05 TS) or 2 (tcgen05 SS)");
  const int warps = n_or_warps, chains = acc_or_chains, iters = 4096;
  if (warps < 1 || warps > 32 || (chains != 1 && chains != 2 && chains != 4 && chains != 8))
    return probe_fail("mma.sync rate: 1..32 warps, 1/2/4/8 chains");
  float* sink = nullptr;
  unsigned long long* dv = nullptr;   // per-CTA cycles
  if (cudaMalloc(&sink, static_cast<size_t>(n_sms) * 1024 * sizeof(float)) != cudaSuccess ||
      cudaMalloc(&dv, static_cast<size_t>(n_sms) * sizeof(unsigned long long)) != cudaSuccess) {
    cudaFree(sink);
    return probe_fail("allocation failed");
  }
  cudaError_t e = cudaSuccess;
  for (int rep = 0; rep < 2 && e == cudaSuccess; ++rep) {
    switch (chains) {
      case 1: hmma_rate_kernel<1><<<n_sms, warps * 32, 0, st>>>(iters, sink, dv); break;
      case 2: hmma_rate_kernel<2><<<n_sms, warps * 32, 0, st>>>(iters, sink, dv); break;
      case 4: hmma_rate_kernel<4><<<n_sms, warps * 32, 0, st>>>(iters, sink, dv); break;
      default: hmma_rate_kernel<8><<<n_sms, warps * 32, 0, st>>>(iters, sink, dv); break;
    }
    e = cudaStreamSynchronize(st);
  }
  std::vector<unsigned long long> h(n_sms);
  if (e == cudaSuccess) e = cudaMemcpy(h.data(), dv, n_sms * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  double c = 0;
  for (auto v : h) c += static_cast<double>(v);
  *result = c / n_sms / (static_cast<double>(iters) * chains * warps);   // cycles per MMA per SM
  cudaFree(sink);
  cudaFree(dv);
  if (e != cudaSuccess) return probe_fail(cudaGetErrorString(e));
  return 0;
}

// Per-launch floor of a CUDA graph: a chain of 200 empty dependent kernels of
// n_ctas CTAs x 256 threads (with programmatic dependent launch if pdl),
// replayed 20 times; *us_per_launch = device time per launch.
PROBE_API int probe_launch_floor(int device, int n_ctas, int pdl, double* us_per_launch) {
  using namespace alm;
  if (!us_per_launch || n_ctas < 1 || n_ctas > 4096) return probe_fail("bad argument");
  ProbeStream ps(device);
  if (ps.e != cudaSuccess) return probe_fail(cudaGetErrorString(ps.e));
  cudaStream_t st = ps.st;
  constexpr int kChain = 200, kReps = 20;
  unsigned* word = nullptr;
  if (cudaMalloc(&word, sizeof(unsigned)) != cudaSuccess) return probe_fail("allocation failed");
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cudaError_t e = cudaMemsetAsync(word, 0, sizeof(unsigned), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
  if (e == cudaSuccess) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_ctas, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t le = cudaSuccess;
    for (int i = 0; i < kChain && le == cudaSuccess; ++i) le = cudaLaunchKernelEx(&cfg, nop_chain_kernel, word);
    e = cudaStreamEndCapture(st, &graph);
    if (e == cudaSuccess) e = le;
  }
  if (e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
  if (e == cudaSuccess) e = cudaEventCreate(&e0);
  if (e == cudaSuccess) e = cudaEventCreate(&e1);
  for (int w = 0; w < 3 && e == cudaSuccess; ++w) e = cudaGraphLaunch(exec, st);
  if (e == cudaSuccess) e = cudaEventRecord(e0, st);
  for (int r = 0; r < kReps && e == cudaSuccess; ++r) e = cudaGraphLaunch(exec, st);
  if (e == cudaSuccess) e = cudaEventRecord(e1, st);
  if (e == cudaSuccess) e = cudaEventSynchronize(e1);
  float ms = 0.f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
  *us_per_launch = static_cast<double>(ms) * 1000.0 / (kChain * kReps);
  if (exec) cudaGraphExecDestroy(exec);
  if (graph) cudaGraphDestroy(graph);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaFree(word);
  if (e != cudaSuccess) return probe_fail(cudaGetErrorString(e));
  return 0;
}
