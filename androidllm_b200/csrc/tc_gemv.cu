// Dequant-GEMV on the 5th-generation tensor cores: y(M, N) = x(M, K) . W(N, K)^T
// for M <= 16 activation rows, W in the row-record layout (kernels.cuh).
//
// One CTA covers 128 weight rows (one tcgen05 MMA tile, M = 128) over its K
// range, with `wg` warpgroups, each of four decoding warps and one issuing
// warp:
//   * every decoding warp streams the records of its 32 rows (one tensor-
//     memory lane quarter) through a ring of bulk copies (TMA engine,
//     mbarrier completion, L2 evict-first), exactly like the tile-layout
//     GEMV;
//   * each thread owns one weight row: it decodes the row's 64 codes of a
//     k-block to exact fp16 weights (the operations of the tile layout, so
//     the weights equal androidllm's fp16(f32(q) * f32(scale))) and writes
//     them to a tensor-memory A slot with one tcgen05.st (32 columns);
//   * warpgroup g takes a contiguous run of the CTA's k-blocks and owns three
//     A slots; after its four warps have stored a k-block, its issuing thread
//     runs four tcgen05.mma (M 128, N 16, K 16) from that slot against the
//     activations staged in shared memory, accumulating in the warpgroup's
//     own tensor-memory accumulator, and tcgen05.commit frees the slot when
//     the MMAs have read it.  An issuing thread completes about one MMA per
//     110 ns whatever N is, and issuing threads run concurrently, so each
//     warpgroup issues its own;
//   * each accumulator sums its k-blocks in order, the accumulators are added
//     in warpgroup order, and every output column depends only on its own
//     activation row, so a pass of M rows reproduces M single-row passes bit
//     for bit;
//   * the accumulator is read back with tcgen05.ld (thread = row); K splits
//     across CTAs are summed in split order by the last CTA of a row block;
//     then the fused epilogues of the tile-layout GEMV (STORE, RESID,
//     SWIGLU, LOGITS) run on the thread-per-row values.
// The tensor core takes the contraction off the CUDA cores, which then only
// decode: on B200 the legacy mma.sync path was the limit of the int4 GEMV.
//
// Activations are staged once per CTA as K-major "core matrices" of 8 rows x
// 8 fp16: chunk q (8 columns) of row m at (q * xrows + m) * 16 bytes with
// xrows = 8 for M <= 8 (rows 8..15 of an N = 16 MMA then read the next chunk:
// finite values whose output columns are never stored) or 16.
#include <cudaTypedefs.h>

#include <algorithm>

#include "act.cuh"
#include "kernels.cuh"
#include "repack.cuh"
#include "tc.cuh"

namespace alm {

constexpr int kTcN = 16;              // MMA N of the fused GEMV: activation rows, padded
constexpr int kTcMaxN = 256;          // MMA N of the dense path (STORE, up to 256 rows)
constexpr int kTcMaxWg = 4;           // decoding warpgroups per CTA
constexpr int kTcMaxThreads = 32 * 5 * kTcMaxWg;   // per warpgroup: 4 decoding warps + 1 issuing warp
constexpr int kTcRingSlots = 3;       // weight ring slots per decoding warp
constexpr int kTcAPerWg = 3;          // tensor-memory A slots per warpgroup
constexpr int kTcSlotCols = 32;       // A slot: one k-block of fp16 pairs
constexpr size_t kTcMaxSmem = 225 * 1024;
constexpr int kTcStageBatch = 4;

template <int BITS>
struct TcFmt;
template <>
struct TcFmt<4> { static constexpr int kParts = 2, kItems = 2; };
template <>
struct TcFmt<8> { static constexpr int kParts = 4, kItems = 1; };

__host__ __device__ inline int tc_parts(int bits) { return bits == 4 ? 2 : 4; }
__host__ __device__ inline int tc_items(int bits) { return bits == 4 ? 2 : 1; }
__host__ __device__ inline int tc_rec_bytes(int bits) { return tc_parts(bits) * 512 + 64; }
__host__ __device__ inline int tc_slot_bytes(int bits) { return tc_items(bits) * tc_rec_bytes(bits); }
__host__ __device__ inline int tc_threads(int wg) { return 32 * 5 * wg; }
__host__ __device__ inline int tc_dcol(int wg) { return kTcAPerWg * wg * kTcSlotCols; }
// MMA N for `rows` activation rows, and the rows staged per 8-column chunk
// (8 for M <= 8: the MMA's rows 8..15 then read the next chunk).
__host__ __device__ inline int tc_n(int rows) { return rows <= kTcN ? kTcN : (rows + 15) / 16 * 16; }
__host__ __device__ inline int tc_xrows(int rows) { return rows <= 8 ? 8 : tc_n(rows); }
// A slots, then one accumulator of tc_n(rows) columns per warpgroup.
__host__ __device__ inline int tc_tmem_cols(int wg, int rows) {
  int c = 32;
  while (c < tc_dcol(wg) + wg * tc_n(rows)) c *= 2;
  return c;
}
__host__ __device__ inline size_t tc_stage_bytes(const QTile& w, int rows) {
  const int nkb = w.kps < w.k_blocks ? w.kps : w.k_blocks;
  return static_cast<size_t>(nkb) * 8 * tc_xrows(rows) * 16 + 128;
}
__host__ __device__ inline size_t tc_ring_bytes(const QTile& w) {
  return static_cast<size_t>(4 * w.wg) * kTcRingSlots * tc_slot_bytes(w.bits);
}
size_t tc_gemv_smem_bytes(const QTile& w, int rows) { return tc_stage_bytes(w, rows) + tc_ring_bytes(w); }

// Launch shape for `rows` activation rows.  Up to 16 rows: the weight's own
// split.  Dense (more rows): one decoding warpgroup (the MMAs bound the time)
// and K split across CTAs so the staged activations fit in shared memory.
QTile tc_launch_shape(const QTile& w, int rows) {
  if (rows <= kTcN) return w;
  QTile d = w;
  d.wg = 1;
  const size_t per_kb = static_cast<size_t>(8) * tc_xrows(rows) * 16;
  const size_t budget = kTcMaxSmem - tc_ring_bytes(d) - 1024;
  int kps = static_cast<int>(std::max<size_t>(1, std::min<size_t>(d.k_blocks, budget / per_kb)));
  d.ksg = (d.k_blocks + kps - 1) / kps;
  d.kps = (d.k_blocks + d.ksg - 1) / d.ksg;
  return d;
}

// Launch shape of the dense path with streamed activations: the weight's own
// K split, one decoding warpgroup.
QTile tc_stream_shape(const QTile& w) {
  QTile d = w;
  d.wg = 1;
  return d;
}

size_t tc_part_floats(const QTile& w, int rows) {
  size_t need = 0;
  for (const QTile& d : {tc_launch_shape(w, rows), rows > kTcN ? tc_stream_shape(w) : w})
    if (d.ksg > 1) need = std::max(need, static_cast<size_t>(d.ksg) * tc_n(rows) * d.n_rb * kRowBlock);
  return need;
}

namespace {

struct TcShared {
  uint64_t full[kTcAPerWg * kTcMaxWg];    // A slot stored (4 warp arrivals)
  uint64_t empty[kTcAPerWg * kTcMaxWg];   // A slot read by its MMAs (commit)
  uint64_t dready;                        // every MMA done (one commit per issuing thread)
  uint64_t ring[4 * kTcMaxWg][kTcRingSlots];
  uint32_t tmem;
  int broken;                             // a bounded wait gave up: everyone stops waiting
  int last;
  float den_in[kMaxRows];
  float den_res[kMaxRows];
  float am_v[4][kMaxRows];
  int am_i[4][kMaxRows];
};

// Bounded mbarrier wait that also gives up once another thread has.
ALM_DEV bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* broken) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (unsigned i = 1; i < kSpinLimit; ++i) {
    if (mbar_try_wait_suspend(bar, parity)) return true;
    if (*broken) return false;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  *broken = 1;
  return false;
}

// int4 part (32 codes of one row) -> 16 tensor-memory columns, scaled by s2.
ALM_DEV void tc_decode4(const uint4& q, half2 s2, uint32_t* out) {
  const uint32_t ws[4] = {q.x, q.y, q.z, q.w};
  const half2 off = u2h(0x64086408u);         // 1032 = 1024 + 8
  const half2 sixteenth = u2h(0x2c002c00u);   // 1/16
  const half2 off16 = u2h(0xd480d480u);       // -72 = -(64 + 8)
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t w = ws[j], w8 = w >> 8;
    out[4 * j + 0] = h2u(__hmul2(__hsub2(u2h(and_or(w, 0x000f000fu, 0x64006400u)), off), s2));
    out[4 * j + 1] = h2u(__hmul2(__hfma2(u2h(and_or(w, 0x00f000f0u, 0x64006400u)), sixteenth, off16), s2));
    out[4 * j + 2] = h2u(__hmul2(__hsub2(u2h(and_or(w8, 0x000f000fu, 0x64006400u)), off), s2));
    out[4 * j + 3] = h2u(__hmul2(__hfma2(u2h(and_or(w8, 0x00f000f0u, 0x64006400u)), sixteenth, off16), s2));
  }
}

// int8 part (16 codes of one row) -> 8 tensor-memory columns.
ALM_DEV void tc_decode8(const uint4& q, half2 s2, uint32_t* out) {
  const uint32_t ws[4] = {q.x, q.y, q.z, q.w};
  const half2 off = u2h(0x64806480u);         // 1152 = 1024 + 128
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    out[2 * j] = h2u(__hmul2(__hsub2(u2h(prmt(ws[j], 0x64646464u, 0x4140u)), off), s2));
    out[2 * j + 1] = h2u(__hmul2(__hsub2(u2h(prmt(ws[j], 0x64646464u, 0x4342u)), off), s2));
  }
}

template <int BITS>
ALM_DEV void tc_decode_record(const unsigned char* rec, int lane, uint32_t (&v)[32]) {
  constexpr int P = TcFmt<BITS>::kParts;
  uint4 q[P];
#pragma unroll
  for (int p = 0; p < P; ++p) q[p] = lds128(rec + p * 512 + lane * 16);
  const half s = *reinterpret_cast<const half*>(rec + P * 512 + lane * 2);
  const half2 s2 = __half2half2(s);
#pragma unroll
  for (int p = 0; p < P; ++p) {
    if constexpr (BITS == 4) tc_decode4(q[p], s2, v + 16 * p);
    else tc_decode8(q[p], s2, v + 8 * p);
  }
}

// One decoding warp's weight stream: its records through a ring of bulk
// copies (TMA engine, mbarrier completion, L2 evict-first).
template <int BITS>
struct TcWeightStream {
  static constexpr int IPS = TcFmt<BITS>::kItems;
  static constexpr int REC = TcFmt<BITS>::kParts * 512 + 64;
  static constexpr int SLOT = IPS * REC;
  unsigned char* ring = nullptr;
  uint64_t* bar = nullptr;
  const unsigned char* src = nullptr;
  int cnt = 0;        // records (k-blocks)
  int n_chunks = 0;   // ring chunks of IPS records
  // lane 0: chunk c into ring slot c % kTcRingSlots
  ALM_DEV void issue(int c) const {
    const int slot = c % kTcRingSlots;
    const uint32_t bytes = static_cast<uint32_t>(min(IPS, cnt - c * IPS) * REC);
    mbar_expect_tx(&bar[slot], bytes);
    bulk_g2s(ring + slot * SLOT, src + static_cast<size_t>(c) * IPS * REC, bytes, &bar[slot], l2_evict_first());
  }
  // lane 0: the first chunks (weights do not depend on earlier kernels)
  ALM_DEV int issue_first() const {
    for (int c = 0; c < n_chunks && c < kTcRingSlots; ++c) issue(c);
    return min(n_chunks, kTcRingSlots);
  }
};

// A decoding warp: decode its j-th record to exact fp16 rows and store them
// with tcgen05.st into A slot g + wg * (j % NA) (lanes of a_base); arrive on
// full[slot] once stored, wait on empty[slot] (the MMAs that read the slot's
// previous contents) before storing again.  The store of record j completes
// while record j + 1 is decoded.  On a wait that gives up: report it and let
// every copy in flight land before the CTA's shared memory is released.
template <int BITS, int NA = kTcAPerWg>
ALM_DEV void tc_decode_warp(const TcWeightStream<BITS>& ws, int issued, uint32_t a_base, int g, int wg,
                            uint64_t* full, uint64_t* empty, volatile int* broken, int lane, int* err) {
  constexpr int IPS = TcWeightStream<BITS>::IPS, REC = TcWeightStream<BITS>::REC;
  constexpr int SLOT = TcWeightStream<BITS>::SLOT;
  int rslot = 0;
  uint32_t rphase = 0;
  int waited = 0, stored = 0;
  bool ok = true;
  for (int j = 0; j < ws.cnt; ++j) {
    const int jj = j % IPS, c = j / IPS;
    if (jj == 0) {
      ok = __all_sync(0xffffffffu, tc_wait(&ws.bar[rslot], rphase, broken));
      if (!ok) break;
      waited = c + 1;
    }
    uint32_t v[32];
    tc_decode_record<BITS>(ws.ring + rslot * SLOT + jj * REC, lane, v);
    if (j > 0) {
      // the previous k-block's store finished while this one was decoded
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[g + wg * ((j - 1) % NA)]);
    }
    const int aslot = g + wg * (j % NA);
    const int use = j / NA;
    if (use >= 1) {
      ok = __all_sync(0xffffffffu, tc_wait(&empty[aslot], (use - 1) & 1, broken));
      if (!ok) break;
      tc_fence_after();
    }
    __syncwarp();
    tc_st32(a_base + aslot * kTcSlotCols, v);
    stored = j + 1;
    if (jj == IPS - 1 || j == ws.cnt - 1) {
      // the ring slot's reads are complete (their values went through tcgen05.st)
      if (lane == 0 && c + kTcRingSlots < ws.n_chunks) {
        fence_proxy_async_smem();
        ws.issue(c + kTcRingSlots);
        ++issued;
      }
      if (++rslot == kTcRingSlots) {
        rslot = 0;
        rphase ^= 1u;
      }
    }
  }
  if (stored > 0) {
    tc_wait_st();
    tc_fence_before();
    __syncwarp();
    if (ok && lane == 0) mbar_arrive(&full[g + wg * ((stored - 1) % NA)]);
  }
  if (!ok) {
    if (lane == 0 && err) atomicExch(err, 2);
    issued = __shfl_sync(0xffffffffu, issued, 0);
    for (int c = waited; c < issued; ++c) mbar_wait(&ws.bar[c % kTcRingSlots], (c / kTcRingSlots) & 1u);
  }
}

// Dense store epilogue (more than 16 rows): the n_acc accumulators (N =
// tc_n(M) columns each, from dlane) read 16 activation rows at a time and
// added in accumulator order; with K split across
// CTAs, row-major partials part[(split * rows_pad + row) * n_mma + m] (a
// thread moves its row's values as independent 16-byte accesses), summed in
// split order by the last CTA of the row block.  All threads of the CTA call
// it (block barriers); warps 0-3 hold the rows.
ALM_DEV void tc_dense_store(const QTile& w, int rb, int ks, int M, uint32_t dlane, int n_acc, half* out, int ldo,
                            int n_out, float* __restrict__ part, int* s_last) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = rb * kRowBlock + warp * 32 + lane;
  const size_t rows_pad = static_cast<size_t>(w.n_rb) * kRowBlock;
  const int n_mma = tc_n(M);
  const bool valid = row < n_out;
  if (warp < 4) {
    for (int q = 0; q < n_mma / 16; ++q) {
      uint32_t d[16];
      tc_ld16(dlane + 16 * q, d);
      tc_wait_ld();
      for (int a = 1; a < n_acc; ++a) {
        uint32_t e[16];
        tc_ld16(dlane + a * n_mma + 16 * q, e);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) d[i] = __float_as_uint(fadd(__uint_as_float(d[i]), __uint_as_float(e[i])));
      }
      if (w.ksg > 1) {
        float4* dst = reinterpret_cast<float4*>(part + (static_cast<size_t>(ks) * rows_pad + row) * n_mma + 16 * q);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          dst[i] = make_float4(__uint_as_float(d[4 * i]), __uint_as_float(d[4 * i + 1]),
                               __uint_as_float(d[4 * i + 2]), __uint_as_float(d[4 * i + 3]));
      } else {
#pragma unroll
        for (int mm = 0; mm < 16; ++mm) {
          const int m = 16 * q + mm;
          if (m < M && valid) out[static_cast<size_t>(m) * ldo + row] = __float2half_rn(__uint_as_float(d[mm]));
        }
      }
    }
  }
  if (w.ksg > 1) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *s_last = atomicAdd(&w.counters[rb], 1u) == static_cast<unsigned>(w.ksg - 1);
    __syncthreads();
    if (*s_last) {
      __threadfence();
      if (warp < 4 && valid)
        for (int q = 0; q < n_mma / 16; ++q) {
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.f;
          // splits summed in order; four splits' loads in flight at a time
          for (int sp0 = 0; sp0 < w.ksg; sp0 += 4) {
            float4 ld[4][4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int sp = sp0 + j;
              const float4* src = reinterpret_cast<const float4*>(
                  part + (static_cast<size_t>(sp < w.ksg ? sp : 0) * rows_pad + row) * n_mma + 16 * q);
#pragma unroll
              for (int i = 0; i < 4; ++i) ld[j][i] = sp < w.ksg ? __ldcg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if (sp0 + j >= w.ksg) break;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                v[4 * i] = fadd(v[4 * i], ld[j][i].x);
                v[4 * i + 1] = fadd(v[4 * i + 1], ld[j][i].y);
                v[4 * i + 2] = fadd(v[4 * i + 2], ld[j][i].z);
                v[4 * i + 3] = fadd(v[4 * i + 3], ld[j][i].w);
              }
            }
          }
#pragma unroll
          for (int mm = 0; mm < 16; ++mm) {
            const int m = 16 * q + mm;
            if (m < M) out[static_cast<size_t>(m) * ldo + row] = __float2half_rn(v[mm]);
          }
        }
      if (threadIdx.x == 0) atomicExch(&w.counters[rb], 0u);
    }
  }
}

template <int BITS, int EPI>
__global__ void __launch_bounds__(kTcMaxThreads, 1)
    tc_gemv_kernel(const __grid_constant__ QTile w, const __grid_constant__ ActIn in, int M,
                   const __grid_constant__ Epi epi, StepIO io, float* __restrict__ part) {
  constexpr int IPS = TcFmt<BITS>::kItems;
  constexpr int REC = TcFmt<BITS>::kParts * 512 + 64;
  constexpr int SLOT = IPS * REC;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ TcShared sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_warps = blockDim.x >> 5;
  const int wg = w.wg, n_dec = 4 * wg;
  const bool decoder = warp < n_dec;
  const int rb = blockIdx.x, ks = blockIdx.y;
  const int cta_kb0 = ks * w.kps;
  const int nkb = max(0, min(w.kps, w.k_blocks - cta_kb0));
  const int per = (nkb + wg - 1) / wg;
  const int xrows = tc_xrows(M);
  uint4* xs = reinterpret_cast<uint4*>(smem);
  unsigned char* rings = smem + tc_stage_bytes(w, M);

  // ---- set-up: barriers, tensor memory ---------------------------------------
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcAPerWg * wg; ++i) {
      mbar_init(&sh.full[i], 4);
      mbar_init(&sh.empty[i], 1);
    }
    mbar_init(&sh.dready, wg);
    sh.broken = 0;
  }
  if (decoder && lane == 0)
    for (int i = 0; i < kTcRingSlots; ++i) mbar_init(&sh.ring[warp][i], 1);
  if (lane == 0) fence_mbar_init();
  if (warp == n_dec) tc_alloc(&sh.tmem, tc_tmem_cols(wg, M));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;

  // ---- weight stream of this warp (independent of earlier kernels) -----------
  const int g = warp >> 2, grp = warp & 3;
  const int my0 = g * per;
  const int cnt = decoder ? max(0, min(per, nkb - my0)) : 0;
  const int n_chunks = (cnt + IPS - 1) / IPS;
  TcWeightStream<BITS> ws;
  ws.src = reinterpret_cast<const unsigned char*>(
      w.data + (static_cast<size_t>(rb * 4 + grp) * w.k_blocks + cta_kb0 + my0) * w.rec_u4);
  ws.ring = rings + static_cast<size_t>(decoder ? warp : 0) * kTcRingSlots * SLOT;
  ws.bar = sh.ring[decoder ? warp : 0];
  ws.cnt = cnt;
  ws.n_chunks = n_chunks;
  int issued = 0;
  if (decoder && lane == 0) issued = ws.issue_first();

  grid_dep_wait();

  // ---- deferred-norm denominators --------------------------------------------
  for (int m = warp; m < M; m += n_warps) {
    if (in.ss) {
      const float d = row_denominator(in, m);
      if (lane == 0) sh.den_in[m] = d;
    }
    if constexpr (EPI == EPI_RESID) {
      if (epi.res.ss) {
        const float d = row_denominator(epi.res, m);
        if (lane == 0) sh.den_res[m] = d;
      }
    }
  }
  __syncthreads();

  // ---- activations -> shared memory (MMA B operand) --------------------------
  if (M > kTcN && in.ss == nullptr && in.vec) {
    // dense path, raw rows: asynchronous 16-byte copies, coalesced along K
    // (padding rows and columns past k_real read as zeros)
    // a warp covers 8 rows x 4 chunks: 64 contiguous bytes of each row from
    // global memory, 4 runs of 128 contiguous bytes in shared memory
    const int per_row = nkb * 8;
    const int n_stage = per_row * xrows;
    for (int c = threadIdx.x; c < n_stage; c += blockDim.x) {
      const int mi = c & 7, qi = (c >> 3) & 3, rest = c >> 5;
      const int q = (rest % (per_row / 4)) * 4 + qi, m = (rest / (per_row / 4)) * 8 + mi;
      const int col0 = cta_kb0 * 64 + q * 8;
      const int valid = m < M ? max(0, min(8, w.k_real - col0)) : 0;
      const half* src = in.x + static_cast<size_t>(valid ? m : 0) * in.ld + (valid ? col0 : 0);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(xs + q * xrows + m)), "l"(src),
                   "r"(valid * 2)
                   : "memory");
    }
    if (threadIdx.x < 8) xs[n_stage + threadIdx.x] = make_uint4(0, 0, 0, 0);
    asm volatile("cp.async.commit_group;\n cp.async.wait_group 0;" ::: "memory");
    fence_proxy_async_smem();
  } else {
    const int per_row = nkb * 8;
    const int n_stage = per_row * xrows;   // padding rows are zeroed
    const bool deferred = in.ss != nullptr;
    for (int base = 0; base < n_stage; base += blockDim.x * kTcStageBatch) {
      uint4 raw[kTcStageBatch], wv[kTcStageBatch];
#pragma unroll
      for (int j = 0; j < kTcStageBatch; ++j) {
        const int c = base + j * blockDim.x + threadIdx.x;
        const int m = c % xrows, q = c / xrows;
        const int col0 = cta_kb0 * 64 + q * 8;
        const bool ok = c < n_stage && m < M;
        raw[j] = ok ? load_row8(in, m, col0, w.k_real) : make_uint4(0, 0, 0, 0);
        wv[j] = (ok && deferred) ? load_w8(in.w, col0, w.k_real, in.vec) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < kTcStageBatch; ++j) {
        const int c = base + j * blockDim.x + threadIdx.x;
        if (c >= n_stage) break;
        const int m = c % xrows;
        uint4 v = raw[j];
        if (deferred && m < M) {
          const float den = sh.den_in[m];
          uint32_t words[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float a0 = norm_value(u4_half(raw[j], 2 * e), den, u4_half(wv[j], 2 * e));
            const float a1 = norm_value(u4_half(raw[j], 2 * e + 1), den, u4_half(wv[j], 2 * e + 1));
            words[e] = h2u(__floats2half2_rn(a0, a1));
          }
          v = make_uint4(words[0], words[1], words[2], words[3]);
        }
        xs[c] = v;   // c = q * xrows + m
      }
    }
    if (threadIdx.x < 8) xs[n_stage + threadIdx.x] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();   // generic-proxy writes, read by the tensor core
  }
  __syncthreads();

  // ---- decoding warps: records -> exact fp16 rows -> tensor memory -----------
  if (decoder) {
    tc_decode_warp<BITS>(ws, issued, tmem + (static_cast<uint32_t>(grp * 32) << 16), g, wg, sh.full, sh.empty,
                         &sh.broken, lane, io.err);
  } else if (lane == 0) {
    // ---- issuing thread of warpgroup gi: its k-blocks in order, own accumulator --
    const int gi = warp - n_dec;
    const int cg = max(0, min(per, nkb - gi * per));
    const uint32_t idesc = tc_idesc_f16(kRowBlock, tc_n(M));
    const uint32_t dcol = tmem + tc_dcol(wg) + gi * tc_n(M);
    const uint32_t xbase = smem_addr(xs);
    const uint32_t lbo = static_cast<uint32_t>(xrows) * 16;
    bool ok = true;
    for (int j = 0; j < cg; ++j) {
      const int aslot = gi + wg * (j % kTcAPerWg);
      if (!(ok = tc_wait(&sh.full[aslot], (j / kTcAPerWg) & 1, &sh.broken))) break;
      tc_fence_after();
      const int kbl = gi * per + j;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint64_t bd = tc_sdesc(xbase + static_cast<uint32_t>((kbl * 8 + 2 * s) * xrows * 16), lbo, 128);
        tc_mma_ts(dcol, tmem + aslot * kTcSlotCols + 8 * s, bd, idesc, j > 0 || s > 0);
      }
      tc_commit(&sh.empty[aslot]);
    }
    tc_commit(&sh.dready);
    if (!ok) {
      if (io.err) atomicExch(io.err, 2);
      mbar_wait(&sh.dready, 0);   // the MMAs issued so far finish before tensor memory is freed
    }
  }

  // ---- accumulator -> registers (thread = row) ---------------------------------
  float acc[kTcN];
#pragma unroll
  for (int n = 0; n < kTcN; ++n) acc[n] = 0.f;
  const int r_local = warp * 32 + lane;
  const int row = rb * kRowBlock + r_local;
  const uint32_t dlane = tmem + (static_cast<uint32_t>(warp * 32) << 16) + tc_dcol(wg);
  if (warp < 4) {
    const bool ok = __all_sync(0xffffffffu, tc_wait(&sh.dready, 0, &sh.broken));
    tc_fence_after();
    __syncwarp();
    if (M <= kTcN) {
      // warpgroup accumulators summed in warpgroup order (those with k-blocks)
      for (int gi = 0; gi < wg && gi * per < nkb; ++gi) {
        uint32_t d[kTcN];
        tc_ld16(dlane + gi * kTcN, d);
        tc_wait_ld();
#pragma unroll
        for (int n = 0; n < kTcN; ++n) acc[n] = gi == 0 ? __uint_as_float(d[n]) : fadd(acc[n], __uint_as_float(d[n]));
      }
    }
    if (!ok && lane == 0 && io.err) atomicExch(io.err, 2);
  }
  grid_dep_launch();

  bool do_epi = true;
  if (M > kTcN) {
    tc_dense_store(w, rb, ks, M, dlane, 1, epi.out, epi.ldo, epi.n_out, part, &sh.last);
    do_epi = false;
  } else if (w.ksg > 1) {
    // ---- K splits: partials, summed in split order by the last CTA --------------
    const size_t rows_pad = static_cast<size_t>(w.n_rb) * kRowBlock;
    if (warp < 4) {
#pragma unroll
      for (int m = 0; m < kTcN; ++m)
        if (m < M) part[(static_cast<size_t>(ks) * kTcN + m) * rows_pad + row] = acc[m];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) sh.last = atomicAdd(&w.counters[rb], 1u) == static_cast<unsigned>(w.ksg - 1);
    __syncthreads();
    do_epi = sh.last != 0;
    if (do_epi) {
      __threadfence();
      if (warp < 4) {
#pragma unroll
        for (int m = 0; m < kTcN; ++m) {
          if (m >= M) continue;
          float s = 0.f;
          for (int sp = 0; sp < w.ksg; ++sp) s = fadd(s, __ldcg(part + (static_cast<size_t>(sp) * kTcN + m) * rows_pad + row));
          acc[m] = s;
        }
      }
      if (threadIdx.x == 0) atomicExch(&w.counters[rb], 0u);
    }
  }

  // ---- fused epilogues (rounding points of androidllm/models/llama.py:96-146) --
  if (do_epi && warp < 4) {
    const bool valid = row < epi.n_out;
    if constexpr (EPI == EPI_STORE) {
#pragma unroll
      for (int m = 0; m < kTcN; ++m)
        if (m < M && valid) epi.out[static_cast<size_t>(m) * epi.ldo + row] = __float2half_rn(acc[m]);
    } else if constexpr (EPI == EPI_RESID) {
      const ActIn& rs = epi.res;
      const float rw = (rs.ss && valid) ? __half2float(__ldg(rs.w + row)) : 1.f;
#pragma unroll
      for (int m = 0; m < kTcN; ++m) {
        if (m >= M) continue;
        float sf = 0.f;
        if (valid) {
          const float rv = __half2float(__ldcg(rs.x + static_cast<size_t>(m) * rs.ld + row));
          const float o = round_h(acc[m]);
          const float res = rs.ss ? norm_value(rv, sh.den_res[m], rw) : rv;
          const half s16 = __float2half_rn(fadd(res, o));
          epi.out[static_cast<size_t>(m) * epi.ldo + row] = s16;
          sf = __half2float(s16);
        }
        float sq = fmul(sf, sf);
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) sq = fadd(sq, __shfl_xor_sync(0xffffffffu, sq, o));
        const int tile = row >> 4;
        if ((lane & 15) == 0 && tile < w.n_tiles) epi.ss_out[static_cast<size_t>(m) * w.n_tiles + tile] = sq;
      }
    } else if constexpr (EPI == EPI_SWIGLU) {
      // lanes 0-15: gate rows j0 + t, lanes 16-31: up rows j0 + t
      const int col = (rb * 4 + warp) * 16 + (lane & 15);
#pragma unroll
      for (int m = 0; m < kTcN; ++m) {
        if (m >= M) continue;
        const float v = round_h(acc[m]);
        const float uv = __shfl_down_sync(0xffffffffu, v, 16);
        if (lane < 16 && col < epi.n_out) {
          const float sig = fdiv(1.f, fadd(1.f, expf(-v)));
          epi.out[static_cast<size_t>(m) * epi.ldo + col] = __float2half_rn(fmul(fmul(v, sig), uv));
        }
      }
    } else if constexpr (EPI == EPI_LOGITS) {
#pragma unroll
      for (int m = 0; m < kTcN; ++m) {
        if (m >= M) continue;
        float bv = kNegInf;
        int bi = 0x7fffffff;
        if (valid) {
          const half l16 = __float2half_rn(acc[m]);
          epi.out[static_cast<size_t>(m) * epi.ldo + row] = l16;
          bv = __half2float(l16);
          bi = row;
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (lane == 0) {
          sh.am_v[warp][m] = bv;
          sh.am_i[warp][m] = bi;
        }
      }
    }
  }
  if constexpr (EPI == EPI_LOGITS) {
    __syncthreads();
    if (do_epi && threadIdx.x < M) {
      const int m = threadIdx.x;
      float bv = kNegInf;
      int bi = 0x7fffffff;
      for (int k = 0; k < 4; ++k)
        if (better(sh.am_v[k][m], sh.am_i[k][m], bv, bi)) {
          bv = sh.am_v[k][m];
          bi = sh.am_i[k][m];
        }
      epi.am_val[static_cast<size_t>(m) * w.n_rb + rb] = bv;
      epi.am_idx[static_cast<size_t>(m) * w.n_rb + rb] = bi;
    }
  }

  // ---- tear-down -----------------------------------------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == n_dec) {
    __syncwarp();
    tc_dealloc(tmem, tc_tmem_cols(wg, M));
  }
}

// ---------------------------------------------------------------------------
// Dense path with TMA-streamed activations (more than 16 raw rows, 16-byte
// aligned, STORE): one CTA per 128-row block and K split, the activations
// streamed per k-block instead of staged for the whole K range.
//   * A producer thread copies each k-block's activations (64 columns x N
//     rows) with one TMA tensor copy into a ring slot in the canonical
//     K-major SWIZZLE_128B layout (row r at r * 128 bytes, its 16-byte chunk c
//     at c ^ (r % 8)); rows past M and columns past k_real read as zeros.  It
//     waits only for a slot to be released by the MMAs that read it.
//   * Two warpgroups of four decoding warps take the two halves of the
//     CTA's k-blocks (each warp its 32-row lane quarter, its own weight
//     stream); warpgroup h writes its j-th k-block to tensor-memory A slot
//     h + 2 * (j % 3), so three k-blocks per warpgroup are decoded while the
//     MMAs of earlier ones complete.  Producer and issuing threads walk the
//     k-blocks in one interleaved sequence (h0 j0, h1 j0, h0 j1, ...).
//   * n_iss issuing threads take the sequence positions in turn (thread i:
//     q = i, i + n_iss, ...), each into its own tensor-memory accumulator: one
//     issuing thread completes about one MMA per 110 ns for any N, and the
//     SM's tensor pipe is full when the concurrent MMAs add up to N = 256, so
//     n_iss = 4, 2 or 1 as 256 / N allows (a template parameter).  An
//     issuing thread waits for both operands of its k-block, runs the four
//     MMAs (M 128, N = M rounded up to 16, K 16) and commits both slots
//     free.  The accumulators are added in issuer order by the epilogue.
// K is split across CTAs only as the weight's own split says; the splits'
// fp32 partials are summed in split order by tc_split_reduce_kernel.
// ---------------------------------------------------------------------------
constexpr int kTcGemmDec = 8;            // decoding warps (two warpgroups)
constexpr int kTcGemmAPerWg = 3;         // tensor-memory A slots per decoding warpgroup
constexpr int kTcGemmA = 2 * kTcGemmAPerWg;
constexpr int kTcGemmMaxXSlots = 8;      // activation ring slots (fewer for N > 128)
constexpr int kTcGemmMaxIss = 4;         // issuing threads (one per warp)
constexpr int kTcGemmThreads = 32 * (kTcGemmDec + kTcGemmMaxIss + 1);   // at most: decoding, issuing, producer

struct TcGemmShared {
  uint64_t full[kTcGemmA], empty[kTcGemmA];
  uint64_t xfull[kTcGemmMaxXSlots], xempty[kTcGemmMaxXSlots];
  uint64_t dready;
  uint64_t ring[kTcGemmDec][kTcRingSlots];
  uint32_t tmem;
  int broken;
};

// Position q of the interleaved k-block sequence -> (warpgroup h, its j-th
// k-block); warpgroup 1 has cnt1 k-blocks, warpgroup 0 cnt1 or cnt1 + 1.
ALM_DEV void tc_gemm_pos(int q, int cnt1, int& h, int& j) {
  if (q < 2 * cnt1) {
    h = q & 1;
    j = q >> 1;
  } else {
    h = 0;
    j = q - cnt1;
  }
}

// 1, 2 or 4 issuing threads, so that their MMAs add up to at most N = 256.
__host__ __device__ inline int tc_gemm_issuers(int rows) {
  const int n = 256 / tc_n(rows);
  return n >= 4 ? 4 : n >= 2 ? 2 : 1;
}
// Tensor memory: A slots in columns [0, 192), then the issuers' accumulators.
__host__ __device__ constexpr int tc_gemm_dcol() { return kTcGemmA * kTcSlotCols; }
__host__ __device__ inline int tc_gemm_tmem_cols(int rows, int n_iss) {
  int c = 32;
  while (c < tc_gemm_dcol() + n_iss * tc_n(rows)) c *= 2;
  return c;
}
__host__ __device__ inline size_t tc_gemm_ring_bytes(int bits) {
  return static_cast<size_t>(kTcGemmDec) * kTcRingSlots * tc_slot_bytes(bits);
}
__host__ __device__ inline int tc_gemm_xslots(int bits, int rows) {
  const size_t slot = static_cast<size_t>(tc_n(rows)) * 128;
  const size_t n = (kTcMaxSmem - 1024 - tc_gemm_ring_bytes(bits)) / slot;
  return static_cast<int>(n < kTcGemmMaxXSlots ? n : kTcGemmMaxXSlots);
}
// 1024 bytes of slack put the swizzled slots on a 1024-byte boundary.
__host__ __device__ inline size_t tc_gemm_smem_bytes(int bits, int rows) {
  return 1024 + static_cast<size_t>(tc_gemm_xslots(bits, rows)) * tc_n(rows) * 128 + tc_gemm_ring_bytes(bits);
}

// Shared-memory descriptor of a K-major SWIZZLE_128B operand: 8-row groups
// 1024 bytes apart; the leading byte offset is unused by this layout.  A K16
// step inside the 128-byte swizzle span advances the start by 32 bytes.
ALM_DEV uint64_t tc_sdesc_sw128(uint32_t smem_byte_addr) {
  uint64_t d = static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1) << 16;            // LBO 16 bytes (unused)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;    // SBO
  d |= static_cast<uint64_t>(1) << 46;            // descriptor version of sm_100
  d |= static_cast<uint64_t>(2) << 61;            // SWIZZLE_128B
  return d;
}

ALM_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

// Streamed dense epilogue (warps 0-3, thread = row): the n_acc accumulators
// (N = tc_n(M) columns each, from dlane) added in accumulator order; one K
// split stores fp16 outputs, several store fp32 partials
// part[(ks * N + m) * rows_pad + row] (lanes along rows), summed in split
// order by tc_split_reduce_kernel.
ALM_DEV void tc_gemm_store(int rb, int ks, int ksg, int n_rb, int M, uint32_t dlane, int n_acc, half* out, int ldo,
                           int n_out, float* __restrict__ part) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = rb * kRowBlock + warp * 32 + lane;
  const size_t rows_pad = static_cast<size_t>(n_rb) * kRowBlock;
  const int n_mma = tc_n(M);
  for (int q = 0; q < n_mma / 16; ++q) {
    uint32_t d[16];
    tc_ld16(dlane + 16 * q, d);
    tc_wait_ld();
    for (int a = 1; a < n_acc; ++a) {
      uint32_t e[16];
      tc_ld16(dlane + a * n_mma + 16 * q, e);
      tc_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) d[i] = __float_as_uint(fadd(__uint_as_float(d[i]), __uint_as_float(e[i])));
    }
#pragma unroll
    for (int mm = 0; mm < 16; ++mm) {
      const int m = 16 * q + mm;
      if (m >= M) break;
      if (ksg > 1)
        part[(static_cast<size_t>(ks) * n_mma + m) * rows_pad + row] = __uint_as_float(d[mm]);
      else if (row < n_out)
        out[static_cast<size_t>(m) * ldo + row] = __float2half_rn(__uint_as_float(d[mm]));
    }
  }
}

// out[m][row] = fp16(sum of the K splits' partials in split order); one
// thread per (row, m), lanes along rows.
__global__ void __launch_bounds__(256) tc_split_reduce_kernel(const float* __restrict__ part, int ksg, int n_mma,
                                                              int n_rb, int M, int n_out, half* __restrict__ out,
                                                              int ldo) {
  grid_dep_wait();
  grid_dep_launch();
  const int row = blockIdx.x * blockDim.x + threadIdx.x, m = blockIdx.y;
  if (row >= n_out || m >= M) return;
  const size_t rows_pad = static_cast<size_t>(n_rb) * kRowBlock;
  const size_t stride = static_cast<size_t>(n_mma) * rows_pad;
  const float* p = part + static_cast<size_t>(m) * rows_pad + row;
  float sum = 0.f;
  int sp = 0;
  for (; sp + 4 <= ksg; sp += 4) {
    const float v0 = __ldcg(p + sp * stride), v1 = __ldcg(p + (sp + 1) * stride);
    const float v2 = __ldcg(p + (sp + 2) * stride), v3 = __ldcg(p + (sp + 3) * stride);
    sum = fadd(fadd(fadd(fadd(sum, v0), v1), v2), v3);
  }
  for (; sp < ksg; ++sp) sum = fadd(sum, __ldcg(p + sp * stride));
  out[static_cast<size_t>(m) * ldo + row] = __float2half_rn(sum);
}

template <int BITS, int NISS>
__global__ void __launch_bounds__(kTcGemmThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ QTile w, int M,
                   half* __restrict__ out, int ldo, int n_out, StepIO io, float* __restrict__ part) {
  constexpr int IPS = TcFmt<BITS>::kItems;
  constexpr int kIssuer = kTcGemmDec, kProducer = kTcGemmDec + NISS;   // blockDim = 32 * (8 + NISS + 1)
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ TcGemmShared sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rb = blockIdx.x, ks = blockIdx.y;
  const int cta_kb0 = ks * w.kps;
  const int nkb = max(0, min(w.kps, w.k_blocks - cta_kb0));
  const int half0 = (nkb + 1) / 2, cnt1 = nkb - half0;   // k-blocks of warpgroups 0 and 1
  const int n_mma = tc_n(M);
  const int n_xs = tc_gemm_xslots(BITS, M);
  constexpr int n_iss = NISS;   // tc_gemm_issuers(M) or fewer
  const int tcols = tc_gemm_tmem_cols(M, n_iss);
  const uint32_t xslot_bytes = static_cast<uint32_t>(n_mma) * 128;
  unsigned char* xring = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  unsigned char* rings = xring + static_cast<size_t>(n_xs) * xslot_bytes;

  // ---- set-up ---------------------------------------------------------------------
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcGemmA; ++i) {
      mbar_init(&sh.full[i], 4);
      mbar_init(&sh.empty[i], 1);
    }
    for (int i = 0; i < n_xs; ++i) {
      mbar_init(&sh.xfull[i], 1);
      mbar_init(&sh.xempty[i], 1);
    }
    mbar_init(&sh.dready, n_iss);
    sh.broken = 0;
  }
  if (warp < kTcGemmDec && lane == 0)
    for (int i = 0; i < kTcRingSlots; ++i) mbar_init(&sh.ring[warp][i], 1);
  if (warp == kProducer && lane == 0)
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
  if (lane == 0) fence_mbar_init();
  if (warp == kIssuer) tc_alloc(&sh.tmem, tcols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem;

  const int dh = warp >> 2, quarter = warp & 3;   // decoding warps: warpgroup, lane quarter
  TcWeightStream<BITS> ws;
  int issued = 0;
  if (warp < kTcGemmDec) {
    const int kb_off = dh ? half0 : 0;
    ws.src = reinterpret_cast<const unsigned char*>(
        w.data + (static_cast<size_t>(rb * 4 + quarter) * w.k_blocks + cta_kb0 + kb_off) * w.rec_u4);
    ws.ring = rings + static_cast<size_t>(warp) * kTcRingSlots * TcWeightStream<BITS>::SLOT;
    ws.bar = sh.ring[warp];
    ws.cnt = dh ? cnt1 : half0;
    ws.n_chunks = (ws.cnt + IPS - 1) / IPS;
    if (lane == 0) issued = ws.issue_first();
  }

  grid_dep_wait();

  if (warp < kTcGemmDec) {
    tc_decode_warp<BITS, kTcGemmAPerWg>(ws, issued, tmem + (static_cast<uint32_t>(quarter * 32) << 16), dh, 2,
                                        sh.full, sh.empty, &sh.broken, lane, io.err);
  } else if (warp == kProducer) {
    // ---- activations: k-block j -> ring slot j % n_xs -------------------------------
    if (lane == 0) {
      bool ok = true;
      int sent = 0;
      for (int q = 0; q < nkb; ++q) {
        const int xs = q % n_xs, use = q / n_xs;
        if (use >= 1 && !(ok = tc_wait(&sh.xempty[xs], (use - 1) & 1, &sh.broken))) break;
        int h, j;
        tc_gemm_pos(q, cnt1, h, j);
        mbar_expect_tx(&sh.xfull[xs], xslot_bytes);
        tma_load_2d(xring + static_cast<size_t>(xs) * xslot_bytes, &xmap, (cta_kb0 + (h ? half0 : 0) + j) * 64, 0,
                    &sh.xfull[xs]);
        sent = q + 1;
      }
      if (!ok) {
        if (io.err) atomicExch(io.err, 2);
        // the copies still in flight land before the CTA's shared memory goes
        for (int j = max(0, sent - n_xs); j < sent; ++j) mbar_wait(&sh.xfull[j % n_xs], (j / n_xs) & 1);
      }
    }
  } else if (warp - kIssuer < n_iss && lane == 0) {
    // ---- issuing thread i: k-blocks i, i + n_iss, ... into accumulator i ----------
    const int iss = warp - kIssuer;
    const uint32_t idesc = tc_idesc_f16(kRowBlock, n_mma);
    const uint32_t dcol = tmem + tc_gemm_dcol() + iss * n_mma;
    const uint32_t xbase = smem_addr(xring);
    bool ok = true;
    for (int q = iss; q < nkb; q += n_iss) {
      int h, j;
      tc_gemm_pos(q, cnt1, h, j);
      const int aslot = h + 2 * (j % kTcGemmAPerWg), xs = q % n_xs;
      ok = tc_wait(&sh.full[aslot], (j / kTcGemmAPerWg) & 1, &sh.broken) &&
           tc_wait(&sh.xfull[xs], (q / n_xs) & 1, &sh.broken);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < 4; ++s)
        tc_mma_ts(dcol, tmem + aslot * kTcSlotCols + 8 * s,
                  tc_sdesc_sw128(xbase + xs * xslot_bytes + 32u * static_cast<uint32_t>(s)), idesc, q > iss || s > 0);
      tc_commit(&sh.empty[aslot]);
      tc_commit(&sh.xempty[xs]);
    }
    tc_commit(&sh.dready);
    if (!ok) {
      if (io.err) atomicExch(io.err, 2);
      mbar_wait(&sh.dready, 0);   // the MMAs issued so far finish before tensor memory is freed
    }
  }

  // ---- accumulator -> output ---------------------------------------------------------
  const uint32_t dlane = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + tc_gemm_dcol();
  if (warp < 4) {
    const bool ok = __all_sync(0xffffffffu, tc_wait(&sh.dready, 0, &sh.broken));
    tc_fence_after();
    __syncwarp();
    if (!ok && lane == 0 && io.err) atomicExch(io.err, 2);
  }
  grid_dep_launch();
  if (warp < 4) tc_gemm_store(rb, ks, w.ksg, w.n_rb, M, dlane, min(n_iss, nkb), out, ldo, n_out, part);

  tc_fence_before();
  __syncthreads();
  if (warp == kIssuer) {
    __syncwarp();
    tc_dealloc(tmem, tcols);
  }
}

// One thread per (record, row t): that row's codes and scale.
__global__ void repack_rows_kernel(SrcSet s, const int* __restrict__ dst_src_row, int bits, int n_rb,
                                   int k_blocks, int k_pad, int block, int src_nsb, int rec_u4,
                                   uint4* __restrict__ out) {
  const long long gid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long total = static_cast<long long>(n_rb) * 4 * k_blocks * kWarp;
  if (gid >= total) return;
  const int t = static_cast<int>(gid % kWarp);
  const long long rec = gid / kWarp;
  const int kb = static_cast<int>(rec % k_blocks);
  const int row = static_cast<int>(rec / k_blocks) * kWarp + t;
  const int desc = dst_src_row[row];
  const int parts = bits == 4 ? 2 : 4;
  uint4* dst = out + rec * rec_u4;
  for (int p = 0; p < parts; ++p) {
    uint32_t words[4];
    for (int j = 0; j < 4; ++j) {
      uint32_t wv = 0;
      if (bits == 4) {
        for (int i = 0; i < 8; ++i) {
          const int k = kb * 64 + 32 * p + 8 * j + (i < 4 ? 2 * i : 2 * (i - 4) + 1);
          wv |= static_cast<uint32_t>((fetch_code(s, desc, k, bits, k_pad) + 8) & 0xf) << (4 * i);
        }
      } else {
        for (int b = 0; b < 4; ++b) {
          const int k = kb * 64 + 16 * p + 4 * j + b;
          wv |= static_cast<uint32_t>((fetch_code(s, desc, k, bits, k_pad) + 128) & 0xff) << (8 * b);
        }
      }
      words[j] = wv;
    }
    dst[p * kWarp + t] = make_uint4(words[0], words[1], words[2], words[3]);
  }
  const int sbk = (kb * 64) / block;
  const half sc = (desc < 0 || sbk >= src_nsb) ? __ushort_as_half(0)
                                               : s.scale[desc >> 24][static_cast<size_t>(desc & 0xffffff) * src_nsb + sbk];
  reinterpret_cast<half*>(dst + parts * kWarp)[t] = sc;
}

// Decode the row layout back to fp16 rows (out: n_rows x k_real).
template <int BITS>
__global__ void dequant_rows_kernel(QTile w, half* __restrict__ out) {
  const long long gid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long total = static_cast<long long>(w.n_rb) * 4 * w.k_blocks * kWarp;
  if (gid >= total) return;
  const int t = static_cast<int>(gid % kWarp);
  const long long rec = gid / kWarp;
  const int kb = static_cast<int>(rec % w.k_blocks);
  const int row = static_cast<int>(rec / w.k_blocks) * kWarp + t;
  const unsigned char* rp = reinterpret_cast<const unsigned char*>(w.data + rec * w.rec_u4);
  constexpr int P = TcFmt<BITS>::kParts;
  uint4 q[P];
  for (int p = 0; p < P; ++p) q[p] = reinterpret_cast<const uint4*>(rp)[p * kWarp + t];
  const half2 s2 = __half2half2(reinterpret_cast<const half*>(rp + P * 512)[t]);
  uint32_t v[32];
  for (int p = 0; p < P; ++p) {
    if constexpr (BITS == 4) tc_decode4(q[p], s2, v + 16 * p);
    else tc_decode8(q[p], s2, v + 8 * p);
  }
  if (row >= w.n_rows) return;
  half* o = out + static_cast<size_t>(row) * w.k_real;
  for (int c = 0; c < 32; ++c) {
    const int k = kb * 64 + 2 * c;
    const half2 hv = u2h(v[c]);
    if (k < w.k_real) o[k] = __low2half(hv);
    if (k + 1 < w.k_real) o[k + 1] = __high2half(hv);
  }
}

// cuTensorMapEncodeTiled from the driver (resolved once; null if absent).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// Tensor map of M activation rows (k_real fp16 columns, row stride ld) read
// as 64-column x N-row boxes in the SWIZZLE_128B K-major layout; elements
// outside the matrix read as zeros.
bool tc_encode_xmap(CUtensorMap* map, const half* x, int ld, int M, int k_real) {
  const PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k_real), static_cast<cuuint64_t>(M)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * sizeof(half)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(tc_n(M))};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<half*>(x), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BITS, int EPI>
cudaError_t tc_launch_t(const QTile& w_, const ActIn& in, int M, const Epi& epi, const StepIO& io,
                        const SplitScratch& scr, bool pdl, cudaStream_t st) {
  CUtensorMap xmap;
  if (EPI == EPI_STORE && M > kTcN && in.ss == nullptr && in.vec && tc_encode_xmap(&xmap, in.x, in.ld, M, w_.k_real)) {
    // dense, raw aligned rows: activations streamed per k-block by the TMA engine
    const QTile w = tc_stream_shape(w_);
    if (w.ksg > 1 && (scr.part == nullptr || scr.part_floats < tc_part_floats(w_, M))) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(w.n_rb, w.ksg, 1);
    cfg.dynamicSmemBytes = tc_gemm_smem_bytes(BITS, M);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const int n_iss = tc_gemm_issuers(M);
    cfg.blockDim = dim3(32 * (kTcGemmDec + n_iss + 1), 1, 1);
    cudaError_t e =
        n_iss == 4   ? cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BITS, 4>, xmap, w, M, epi.out, epi.ldo, epi.n_out, io, scr.part)
        : n_iss == 2 ? cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BITS, 2>, xmap, w, M, epi.out, epi.ldo, epi.n_out, io, scr.part)
                     : cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BITS, 1>, xmap, w, M, epi.out, epi.ldo, epi.n_out, io, scr.part);
    if (e != cudaSuccess || w.ksg == 1) return e;
    // K splits: partials summed in split order across the whole GPU
    cfg.gridDim = dim3((epi.n_out + 255) / 256, M, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&cfg, tc_split_reduce_kernel, static_cast<const float*>(scr.part), w.ksg, tc_n(M),
                              w.n_rb, M, epi.n_out, epi.out, epi.ldo);
  }
  const QTile w = tc_launch_shape(w_, M);
  if (w.ksg > 1 && (scr.part == nullptr || scr.part_floats < tc_part_floats(w_, M) || w.counters == nullptr))
    return cudaErrorInvalidValue;
  const size_t smem = tc_gemv_smem_bytes(w, M);
  if (smem > kTcMaxSmem || w.wg < 1 || w.wg > kTcMaxWg) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(w.n_rb, w.ksg, 1);
  cfg.blockDim = dim3(tc_threads(w.wg), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, tc_gemv_kernel<BITS, EPI>, w, in, M, epi, io, scr.part);
}

template <int BITS>
cudaError_t tc_dispatch(EpiKind kind, const QTile& w, const ActIn& in, int M, const Epi& epi, const StepIO& io,
                        const SplitScratch& scr, bool pdl, cudaStream_t st) {
  switch (kind) {
    case EPI_STORE: return tc_launch_t<BITS, EPI_STORE>(w, in, M, epi, io, scr, pdl, st);
    case EPI_RESID: return tc_launch_t<BITS, EPI_RESID>(w, in, M, epi, io, scr, pdl, st);
    case EPI_SWIGLU: return tc_launch_t<BITS, EPI_SWIGLU>(w, in, M, epi, io, scr, pdl, st);
    case EPI_LOGITS: return tc_launch_t<BITS, EPI_LOGITS>(w, in, M, epi, io, scr, pdl, st);
    default: return cudaErrorNotSupported;   // QKV projections use the tile layout
  }
}

template <int BITS>
cudaError_t tc_set_attrs() {
  const int v = static_cast<int>(kTcMaxSmem);
  const auto a = cudaFuncAttributeMaxDynamicSharedMemorySize;
  cudaError_t e = cudaFuncSetAttribute(tc_gemv_kernel<BITS, EPI_STORE>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(tc_gemv_kernel<BITS, EPI_RESID>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(tc_gemv_kernel<BITS, EPI_SWIGLU>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(tc_gemv_kernel<BITS, EPI_LOGITS>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(tc_gemm_kernel<BITS, 1>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(tc_gemm_kernel<BITS, 2>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(tc_gemm_kernel<BITS, 4>, a, v);
  return e;
}

}  // namespace

cudaError_t tc_gemv_init_attrs() {
  cudaError_t e = tc_set_attrs<4>();
  if (e == cudaSuccess) e = tc_set_attrs<8>();
  return e;
}

cudaError_t launch_tc_gemv(const QTile& w, const ActIn& in, int M, EpiKind kind, const Epi& epi,
                           const StepIO& io, const SplitScratch& scr, bool pdl, cudaStream_t st) {
  if (M < 1 || w.layout != kLayoutRow) return cudaErrorInvalidValue;
  if (M > (kind == EPI_STORE ? kTcMaxN : kTcN)) return cudaErrorInvalidValue;   // fused epilogues: <= 16 rows
  if (w.bits == 4) return tc_dispatch<4>(kind, w, in, M, epi, io, scr, pdl, st);
  if (w.bits == 8) return tc_dispatch<8>(kind, w, in, M, epi, io, scr, pdl, st);
  return cudaErrorInvalidValue;
}

cudaError_t launch_repack_rows(const void* const* src, const half* const* src_scales, int n_src,
                               const int* dst_src_row, const QTile& w, uint4* data, int k_pad, cudaStream_t st) {
  if (n_src < 1 || n_src > 3 || (w.bits != 4 && w.bits != 8) || w.block % 64 != 0) return cudaErrorInvalidValue;
  SrcSet s{};
  for (int i = 0; i < n_src; ++i) {
    s.data[i] = static_cast<const uint8_t*>(src[i]);
    s.scale[i] = src_scales ? src_scales[i] : nullptr;
  }
  const long long total = static_cast<long long>(w.n_rb) * 4 * w.k_blocks * kWarp;
  const int threads = 256;
  repack_rows_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0, st>>>(
      s, dst_src_row, w.bits, w.n_rb, w.k_blocks, k_pad, w.block, k_pad / w.block, w.rec_u4, data);
  return cudaGetLastError();
}

cudaError_t launch_dequant_rows(const QTile& w, half* out, cudaStream_t st) {
  const long long total = static_cast<long long>(w.n_rb) * 4 * w.k_blocks * kWarp;
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((total + threads - 1) / threads);
  if (w.bits == 4) dequant_rows_kernel<4><<<blocks, threads, 0, st>>>(w, out);
  else if (w.bits == 8) dequant_rows_kernel<8><<<blocks, threads, 0, st>>>(w, out);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace alm
