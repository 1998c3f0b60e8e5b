// Shared device helpers for the androidllm B200 kernels (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define ALM_DEV __device__ __forceinline__

namespace alm {

constexpr int kWarp = 32;
#define kNegInf (-__int_as_float(0x7f800000))

// ---------------------------------------------------------------------------
// loads
// ---------------------------------------------------------------------------
// Weights are streamed once per forward: read-only path, no L1 allocation.
ALM_DEV uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
ALM_DEV uint32_t ld_nc_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

// ---------------------------------------------------------------------------
// bulk copies (TMA engine, each CTA its own copy) into shared memory with mbarriers
// ---------------------------------------------------------------------------
// Limits of every mbarrier wait: after this many polls, or this much time on
// the global timer, the waiter gives up and reports an error instead of
// hanging (a copy of valid memory completes in microseconds).
constexpr unsigned kSpinLimit = 1u << 24;
constexpr unsigned long long kWaitLimitNs = 200ull * 1000 * 1000;
// A waiting thread is suspended in hardware until the phase completes or at
// most this long, so that waiting warps take no issue slots from working ones.
constexpr uint32_t kSuspendNs = 20000;

ALM_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

ALM_DEV uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
ALM_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
ALM_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
ALM_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
ALM_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// L2 policy for data read once per forward (weights): evicted first, so the
// stream does not push activations, the KV cache or kernel code out of L2.
ALM_DEV uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// global -> shared bulk copy; dst, src 16-byte aligned, bytes a multiple of 16
ALM_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
ALM_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// As mbar_try_wait, suspending the thread until the phase completes or
// kSuspendNs have passed.
ALM_DEV bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of `parity`; false if the limit ran out.
ALM_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (unsigned i = 1; i < kSpinLimit; ++i) {
    if (mbar_try_wait_suspend(bar, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) return false;
  }
  return false;
}
// Plain loads: the compiler orders them after a preceding mbarrier wait (its
// asm has a memory clobber) and may schedule them freely otherwise.
ALM_DEV uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }
ALM_DEV uint32_t lds32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Barrier of the 256 threads that run a shared device body (attention, row
// and embedding bodies): the whole block in kernels of 256 threads, warps
// 0-7 (named barrier 1) in kernels that add a weight-producer warp.
ALM_DEV void body_sync() {
  if (blockDim.x == 256) {
    __syncthreads();
  } else {
    asm volatile("bar.sync 1, 256;" ::: "memory");
  }
}

// body_sync with the barrier chosen at compile time (NAMED: named barrier 1
// over warps 0-7; else the whole block), for bodies on the hot path.
template <bool NAMED>
ALM_DEV void body_sync_t() {
  if constexpr (NAMED) {
    asm volatile("bar.sync 1, 256;" ::: "memory");
  } else {
    __syncthreads();
  }
}

// Argmax order: larger value first, then the smaller index.
ALM_DEV bool better(float v1, int i1, float v2, int i2) { return v1 > v2 || (v1 == v2 && i1 < i2); }

// Programmatic dependent launch: wait for the producer grid's results / let
// the next grid in the stream start its prologue.  No-ops without PDL.
ALM_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
ALM_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }
// Where a shared body passes its dependency wait: a standalone kernel gives
// DepWait (the body loads what earlier kernels wrote before it, then waits
// for its producer); persistent kernels, whose phases are ordered by grid
// barriers, give NoWait.
struct NoWait {
  ALM_DEV void operator()() const {}
};
struct DepWait {
  ALM_DEV void operator()() const { grid_dep_wait(); }
};

// ---------------------------------------------------------------------------
// bit tricks for int4/int8 -> fp16 (exact small integers)
// ---------------------------------------------------------------------------
// (a & b) | c in one LOP3.
ALM_DEV uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}
ALM_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
ALM_DEV uint32_t h2u(half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
ALM_DEV half2 u2h(uint32_t u) { return *reinterpret_cast<half2*>(&u); }

// ---------------------------------------------------------------------------
// tensor core: D = A(16x16, row) * B(16x8, col) + D, fp16 in, fp32 accumulate
// A regs: {a0a1: (g, 2t..2t+1)} {a2a3: (g+8, 2t..)} {a4a5: (g, 2t+8..)} {a6a7: (g+8, 2t+8..)}
// B regs: {b0b1: (k=2t..2t+1, n=g)} {b2b3: (k=2t+8.., n=g)}
// D: {d0,d1: (g, 2t..2t+1)} {d2,d3: (g+8, 2t..2t+1)}        g = lane/4, t = lane%4
// ---------------------------------------------------------------------------
ALM_DEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                      uint32_t b0, uint32_t b1) {
  // no side effects: not volatile, so independent MMAs can be interleaved
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

ALM_DEV void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}
ALM_DEV void ldmatrix_x2(uint32_t& r0, uint32_t& r1, const void* p) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1) : "r"(a));
}
ALM_DEV void ldmatrix_x2_trans(uint32_t& r0, uint32_t& r1, const void* p) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1) : "r"(a));
}

// fp32 arithmetic with no contraction, so results match numpy's separately
// rounded operations.
ALM_DEV float fmul(float a, float b) { return __fmul_rn(a, b); }
ALM_DEV float fadd(float a, float b) { return __fadd_rn(a, b); }
ALM_DEV float fsub(float a, float b) { return __fsub_rn(a, b); }
ALM_DEV float fdiv(float a, float b) { return __fdiv_rn(a, b); }
ALM_DEV float round_h(float a) { return __half2float(__float2half_rn(a)); }

// exp(x) for fp32 x <= 0 from correctly rounded fp32 operations only.
ALM_DEV float rexp(float x) {
  const float log2e = __uint_as_float(0x3fb8aa3bu);
  const float ln2_hi = __uint_as_float(0x3f317200u);   // fp32(ln 2) with its low 9 mantissa bits cleared
  const float ln2_lo = __uint_as_float(0x35bfbe8eu);   // fp32(ln 2 - ln2_hi)
  const float k = rintf(fmul(x, log2e));
  const float r = fsub(fsub(x, fmul(k, ln2_hi)), fmul(k, ln2_lo));
  // 1/7!, 1/6!, ..., 1/1!, 1/0! in Horner order
  const uint32_t c[8] = {0x39500d01u, 0x3ab60b61u, 0x3c088889u, 0x3d2aaaabu,
                         0x3e2aaaabu, 0x3f000000u, 0x3f800000u, 0x3f800000u};
  float acc = __uint_as_float(c[0]);
#pragma unroll
  for (int i = 1; i < 8; ++i) acc = fadd(fmul(acc, r), __uint_as_float(c[i]));
  // exact scaling by 2^k: for x >= -87, k >= -126 so 2^k is a normal fp32 and
  // one correctly rounded multiply equals ldexp
  const int ki = static_cast<int>(k);
  const float scale = __int_as_float((ki + 127) << 23);
  return x < __uint_as_float(0xc2ae0000u) ? 0.f : fmul(acc, scale);   // below -87: 0
}


ALM_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
ALM_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace alm
