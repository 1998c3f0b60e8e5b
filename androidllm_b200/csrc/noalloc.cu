// alm_qmatmul_noalloc: the dequant-GEMV with its split-K scratch in a
// fixed-size device array that lives in the library image, for callers that
// must not allocate device memory once they are running.
//
// Who needs it: real-time loops that cannot afford the implicit device
// synchronisation a cudaMalloc/cudaFree may cause, and hosts that give the
// library a fixed memory budget at start-up and forbid driver allocations
// afterwards.
// alm_qmatmul allocates its split-K partial-sum buffer lazily with
// cudaMalloc; this entry point instead uses the array below, whose address is
// resolved once per device.
//
// Limits and sharing:
//   * the array holds kNoAllocPartFloats fp32 partial sums (2 MiB) and
//     kNoAllocCounters column counters; weights whose split needs more are
//     rejected with ALM_ERR_ARG;
//   * every GPU that loads the library reserves this memory until exit;
//   * all calls on a device share the array: calls that can overlap on the
//     GPU (different streams or contexts of one device) race with each other
//     and must be ordered by the caller;
//   * the counters are cleared on the call's stream before each launch (the
//     array keeps whatever the previous call left).
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/androidllm_b200.h"
#include "common.cuh"
#include "kernels.cuh"

namespace {

constexpr size_t kNoAllocPartFloats = 512 * 1024;   // 2 MiB of fp32 partial sums
constexpr size_t kNoAllocCounters = 4096;           // CTA-column counters
constexpr size_t kNoAllocBytes = kNoAllocPartFloats * sizeof(float) + kNoAllocCounters * sizeof(unsigned);

// File-scope scratch.  In host code `g_noalloc_scratch` is only a host-side
// stand-in for the symbol, never a device address: the device address comes
// from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

thread_local std::string g_msg;

}  // namespace

// Defined in runtime.cu: the error reporting shared by every entry point.
struct alm_ctx;
struct alm_qweight;
int alm_internal_fail(int code, const char* msg);
int alm_internal_qweight_tile(const alm_qweight* w, alm::QTile* t, int* out_rows, int* in_real);
int alm_internal_ctx(alm_ctx* ctx, int* device, cudaStream_t* stream);

extern "C" ALM_API int alm_qmatmul_noalloc(alm_ctx* ctx, const alm_qweight* w, const uint16_t* x_dev, int ldx,
                                           int m, uint16_t* y_dev, int ldy) {
  if (!ctx || !w || !x_dev || !y_dev) return alm_internal_fail(ALM_ERR_ARG, "null argument");
  if (m < 1 || m > alm::kMaxRows) return alm_internal_fail(ALM_ERR_ARG, "m must be in 1..16");
  int device = 0;
  cudaStream_t stream = nullptr;
  int rc = alm_internal_ctx(ctx, &device, &stream);
  if (rc) return rc;
  alm::QTile t;
  int out_rows = 0, in_real = 0;
  rc = alm_internal_qweight_tile(w, &t, &out_rows, &in_real);
  if (rc) return rc;
  if (ldx < in_real || ldy < out_rows) return alm_internal_fail(ALM_ERR_ARG, "leading dimension too small");
  if (device < 0 || device >= kMaxDevices) return alm_internal_fail(ALM_ERR_ARG, "device index too large");

  // split-K needs: partial sums and one counter per CTA column
  const size_t need = alm::gemv_part_floats(t);
  const size_t cols = static_cast<size_t>(alm::gemv_out_blocks(t));
  if (need > kNoAllocPartFloats || cols > kNoAllocCounters) {
    g_msg = "weight needs " + std::to_string(need) + " partial floats / " + std::to_string(cols) +
            " counters; the fixed scratch holds " + std::to_string(kNoAllocPartFloats) + " / " +
            std::to_string(kNoAllocCounters);
    return alm_internal_fail(ALM_ERR_ARG, g_msg.c_str());
  }

  // once per device, with that device current: resolve the array's address
  int prev_device = -1;
  if (cudaGetDevice(&prev_device) != cudaSuccess) prev_device = -1;
  struct Restore {
    int d;
    ~Restore() {
      if (d >= 0) cudaSetDevice(d);
    }
  } restore{prev_device};
  if (cudaSetDevice(device) != cudaSuccess) return alm_internal_fail(ALM_ERR_CUDA, "cudaSetDevice failed");
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[device]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) {
        g_msg = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e);
        return alm_internal_fail(ALM_ERR_CUDA, g_msg.c_str());
      }
      g_addr[device] = p;
    }
    base = g_addr[device];
  }
  float* part = static_cast<float*>(base);
  unsigned* counters = reinterpret_cast<unsigned*>(static_cast<unsigned char*>(base) +
                                                   kNoAllocPartFloats * sizeof(float));
  cudaError_t e = cudaMemsetAsync(counters, 0, cols * sizeof(unsigned), stream);
  if (e == cudaSuccess) {
    t.counters = counters;
    alm::Epi epi;
    epi.out = reinterpret_cast<half*>(y_dev);
    epi.ldo = ldy;
    epi.n_out = out_rows;
    alm::ActIn in;
    in.x = reinterpret_cast<const half*>(x_dev);
    in.ld = ldx;
    in.H = in_real;
    e = alm::launch_gemv(t, in, m, alm::EPI_STORE, epi, alm::StepIO{},
                         alm::SplitScratch{part, kNoAllocPartFloats}, false, stream);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) {
    g_msg = std::string("qmatmul_noalloc: ") + cudaGetErrorString(e);
    return alm_internal_fail(ALM_ERR_CUDA, g_msg.c_str());
  }
  return ALM_OK;
}
