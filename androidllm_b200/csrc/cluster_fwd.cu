// Cluster forward: one thread-block cluster of 16 CTAs runs every layer of a
// single-row (decode) forward of a small model, such as the speculative
// draft, in one launch.  Weight streaming and the layer's data dependencies
// are decoupled:
//
//   * a producer warp per CTA streams the CTA's share of every GEMV weight
//     (a contiguous run of qtile records: its output tiles x all k-blocks),
//     layer after layer and projection after projection, through a ring of
//     shared-memory slots with bulk copies (TMA engine, mbarrier completion,
//     each CTA its own copy).  Weights do not depend on activations, so the stream
//     runs ahead across phase boundaries and never waits for them;
//   * eight decoding warps per CTA split the CTA's records into items of
//     (tile, k-split), the weight's own K split of the standalone GEMV (ksw
//     warps x ksg CTAs of kps k-blocks each), decode them with the exact fp16
//     dequant (qtile.cuh) into mma.sync MMAs with the same two accumulator
//     chains, and fold the partial sums in the standalone GEMV's order (the
//     ksw warp partials in order, then the ksg CTA partials in order);
//   * phases (QKV + RoPE + KV write | scores | P.V | O + residual |
//     gate/up + SwiGLU | down + residual) are separated by a cluster barrier
//     of the decoding warps built from distributed-shared-memory mbarrier
//     arrivals, not by kernel boundaries;
//   * attention runs the standalone kernels' device bodies (attn_body.cuh)
//     as virtual blocks over the 16 CTAs.
//
// Every operation, summation order and rounding point is the standalone
// path's (androidllm/models/llama.py:96-128: fp16 matmul outputs of fp32
// sums, RoPE in fp32, fp16 K/V, deferred RMSNorm, SwiGLU in fp32), so a
// cluster forward is bit-identical to the per-operation launches, and a
// single-row decode step stays bit-identical to the same row inside a
// multi-row verify pass.
//
// Every wait is bounded (mbarrier phases, the cluster barrier); a wait that
// gives up sets the error word to 4, later waits of the CTA are skipped, and
// the copies already issued land before the CTA leaves.
#include <mutex>

#include "attn_body.cuh"
#include "cluster_fwd.cuh"
#include "qtile.cuh"
#include "rows_body.cuh"

namespace alm {
namespace {

constexpr int kCfCons = 8;                          // decoding warps
constexpr int kCfConsThreads = kCfCons * kWarp;     // 256: the shared bodies' block
constexpr int kCfThreads = kCfConsThreads + kWarp;  // + the producer warp
constexpr size_t kCfRingBytes = static_cast<size_t>(kCfSlots) * kCfSlotBytes;

struct CfShared {
  uint64_t full[kCfSlots];
  uint64_t empty[kCfSlots];
  uint64_t sync[2];
  float part[kCfMaxItems][16];
  float den_in, den_res;
  volatile int broken;
  AttnShared attn;
};
__shared__ CfShared s_cf;
extern __shared__ __align__(1024) unsigned char s_cf_dyn[];

ALM_DEV unsigned char* cf_work() { return s_cf_dyn + kCfRingBytes; }

ALM_DEV void cons_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

ALM_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %cluster_ctarank;" : "=r"(r));
  return r;
}
ALM_DEV void cluster_barrier_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
ALM_DEV void mbar_arrive_local(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// Arrive on the mbarrier at the same offset in CTA `rank` of the cluster.
ALM_DEV void mbar_arrive_remote(uint64_t* bar, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(bar)), "r"(rank));
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}
// Non-blocking test of a phase with cluster-scope acquire.  The phase sync
// polls with it instead of a suspending try_wait: a thread suspended on a
// barrier is not woken promptly by arrivals from other CTAs (measured: a
// sync then costs up to the whole suspend-time hint).
ALM_DEV bool mbar_test_acq_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Profiling trace (alm_forward_trace): CTA 0 records (label << 48 | global
// ns) at points of its phases into the first half of P.trace (count in
// trace[0]) and its producer lane into the second half (count at trace[half]).
__shared__ int s_cf_tn, s_cf_tp;
ALM_DEV void cf_mark(const FwdParams& P, int label, bool producer = false) {
  if (!P.trace || cluster_rank() != 0) return;
  const int half = P.trace_cap / 2;
  int& n = producer ? s_cf_tp : s_cf_tn;
  unsigned long long* base = P.trace + (producer ? half : 0);
  if (n + 1 < half) base[1 + n++] = (static_cast<unsigned long long>(label) << 48) | (global_ns() & 0xffffffffffffull);
  base[0] = static_cast<unsigned long long>(n);
}

// A wait that gave up: remember it (later waits of this CTA are skipped) and
// report it to the host.
ALM_DEV void cf_fail(const FwdParams& P) {
  s_cf.broken = 1;
  if (P.io.err) atomicExch(P.io.err, 4);
}
// Bounded wait for a phase of one of the CTA's ring barriers, polling with a
// short back-off (no hardware suspension, for the reason above).
ALM_DEV bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
ALM_DEV bool cf_wait(uint64_t* bar, uint32_t parity, const FwdParams& P) {
  if (s_cf.broken) return false;
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (unsigned i = 0; i < (1u << 30); ++i) {
    if (mbar_test(bar, parity)) return true;
    if (i >= 16) __nanosleep(32);
    if ((i & 63) == 63 && global_ns() - t0 > kWaitLimitNs) break;
  }
  cf_fail(P);
  return false;
}

// Cluster barrier of the decoding warps: every consumer thread has finished
// the phase's writes; one thread per CTA arrives on barrier `n & 1` of all 16
// CTAs, then waits (bounded) for the 16 arrivals on its own.  Two barriers
// alternate, so an arrival for the next phase never lands in a phase that is
// still collecting.
ALM_DEV void cf_sync(uint32_t& n, const FwdParams& P) {
  asm volatile("fence.acq_rel.cluster;" ::: "memory");
  cons_sync();
  if (threadIdx.x == 0) {
    uint64_t* bar = &s_cf.sync[n & 1];
    for (uint32_t r = 0; r < kCfCtas; ++r) mbar_arrive_remote(bar, r);
    if (!s_cf.broken) {
      const uint32_t parity = (n >> 1) & 1u;
      const unsigned long long t0 = global_ns();
      bool ok = false;
      for (unsigned i = 0; i < (1u << 30); ++i) {
        if (mbar_test_acq_cluster(bar, parity)) {
          ok = true;
          break;
        }
        if ((i & 255) == 255 && global_ns() - t0 > kWaitLimitNs) break;
      }
      if (!ok) cf_fail(P);
    }
  }
  if (threadIdx.x == 0) cf_mark(P, 6);
  cons_sync();
  ++n;
}

// ---- the CTA's share of one GEMV -----------------------------------------------
ALM_DEV CfPlan cf_plan(const QTile& w, int cta) { return cluster_fwd_plan(w, cta); }

// ---- producer -----------------------------------------------------------------
// Lane 0 of the producer warp streams the chunks of every GEMV phase in
// order; chunk c goes to slot c % kCfSlots once the decoding warps have
// released that slot's previous chunk.
ALM_DEV void cf_produce(const FwdParams& P, int cta) {
  if (threadIdx.x % kWarp != 0) return;
  const uint64_t pol = l2_evict_first();
  uint32_t c = 0;
  bool ok = true;
  for (int li = 0; li < P.n_layers && ok; ++li) {
    const FwdLayer& L = P.layers[li];
    const QTile* ws[4] = {&L.qkv, &L.o, &L.gu, &L.down};
    for (int ph = 0; ph < 4 && ok; ++ph) {
      const CfPlan pl = cf_plan(*ws[ph], cta);
      cf_mark(P, 16 + ph, true);
      for (int k = 0; k < pl.n_chunks; ++k, ++c) {
        const uint32_t slot = c % kCfSlots, use = c / kCfSlots;
        if (use > 0 && !cf_wait(&s_cf.empty[slot], (use - 1) & 1u, P)) {
          ok = false;
          break;
        }
        const int n_rec = min(pl.R, pl.n_rec - k * pl.R);
        const uint32_t bytes = static_cast<uint32_t>(n_rec * pl.rec_bytes);
        fence_proxy_async_smem();
        mbar_expect_tx(&s_cf.full[slot], bytes);
        bulk_g2s(s_cf_dyn + static_cast<size_t>(slot) * kCfSlotBytes,
                 pl.base + static_cast<size_t>(k) * pl.R * pl.rec_bytes, bytes, &s_cf.full[slot], pol);
      }
      cf_mark(P, 32 + ph, true);
    }
  }
  // every issued copy lands before the CTA can leave: the last kCfSlots
  // chunks' full phases (earlier ones were consumed before their slots were
  // reused)
  const uint32_t first = c > static_cast<uint32_t>(kCfSlots) ? c - kCfSlots : 0u;
  for (uint32_t d = first; d < c; ++d) {
    const unsigned long long t0 = global_ns();
    while (!mbar_test(&s_cf.full[d % kCfSlots], (d / kCfSlots) & 1u) && global_ns() - t0 < kWaitLimitNs)
      __nanosleep(32);
  }
}

// ---- decoding warps: one GEMV phase ----------------------------------------------
// Stage the phase input (one row, every k-block) as m16n8k16 B fragments:
// per k-block two halves (k16 steps 0-1, 2-3), per t = lane % 4 one uint4.
ALM_DEV void cf_stage(const QTile& w, const ActIn& in, uint4* xs) {
  uint32_t* xw = reinterpret_cast<uint32_t*>(xs);
  const int per_row = w.k_blocks * 8;   // 8-column chunks
  const bool deferred = in.ss != nullptr;
  const float den = s_cf.den_in;
  for (int c = threadIdx.x; c < per_row; c += kCfConsThreads) {
    const int col0 = c * 8;
    const uint4 raw = load_row8(in, 0, col0, w.k_real);
    uint32_t words[4] = {raw.x, raw.y, raw.z, raw.w};
    if (deferred) {
      const uint4 wv = load_w8(in.w, col0, w.k_real, in.vec);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a0 = norm_value(u4_half(raw, 2 * q), den, u4_half(wv, 2 * q));
        const float a1 = norm_value(u4_half(raw, 2 * q + 1), den, u4_half(wv, 2 * q + 1));
        words[q] = h2u(__floats2half2_rn(a0, a1));
      }
    }
    const int kbl = c / 8, c8 = c % 8;
    const int s = c8 >> 1, hi8 = c8 & 1;
    const int h = s >> 1, r = (s & 1) * 2 + hi8;
#pragma unroll
    for (int tt = 0; tt < 4; ++tt) xw[(((kbl * 2 + h) * 4 + tt) * 4) + r] = words[tt];
  }
}

// Decode and multiply the items of this warp; item partials to s_cf.part.
template <int BITS, int SB>
ALM_DEV void cf_items(const QTile& w, const CfPlan& pl, uint32_t cbase, const uint4* xs, const FwdParams& P) {
  constexpr int V = QTileTraits<BITS>::kVec;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int g = lane >> 2, t = lane & 3;
  const int kbt = w.k_blocks;
  const uint4* xrow = xs + t;
  uint32_t released = cbase;
  for (int j = warp; j < pl.n_items; j += kCfCons) {
    const int tl = j / pl.S, sp = j % pl.S;
    const int kb0 = sp * pl.kps, kb1 = min(kb0 + pl.kps, kbt);
    if (kb0 >= kb1) {   // a split past the last k-block: an exact zero partial
      if (t == 0) s_cf.part[j][g] = s_cf.part[j][g + 8] = 0.f;
      continue;
    }
    const int r0 = tl * kbt + kb0, r1 = tl * kbt + kb1;
    const uint32_t c_first = cbase + static_cast<uint32_t>(r0 / pl.R);
    // chunks before this item's first one are not needed by this warp again
    for (; released < c_first; ++released) {
      __syncwarp();
      if (lane == 0) mbar_arrive_local(&s_cf.empty[released % kCfSlots]);
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t have = 0xffffffffu;   // chunk whose data this warp has waited for
    for (int r = r0; r < r1; ++r) {
      const uint32_t c = cbase + static_cast<uint32_t>(r / pl.R);
      if (c != have) {
        if (!cf_wait(&s_cf.full[c % kCfSlots], (c / kCfSlots) & 1u, P)) break;
        have = c;
      }
      const unsigned char* rp =
          s_cf_dyn + static_cast<size_t>(c % kCfSlots) * kCfSlotBytes + static_cast<size_t>(r % pl.R) * pl.rec_bytes;
      const int kb = r % kbt;
      uint4 cur[V];
#pragma unroll
      for (int v = 0; v < V; ++v) cur[v] = lds128(rp + v * 512 + lane * 16);
      half2 sg_a = __float2half2_rn(1.f), sg8_a = sg_a, sg_b = sg_a, sg8_b = sg_a;
      if constexpr (SB >= 1) {
        const half2 sa = u2h(lds32(rp + V * 512 + g * 4));
        sg_a = __low2half2(sa);
        sg8_a = __high2half2(sa);
        sg_b = sg_a;
        sg8_b = sg8_a;
      }
      if constexpr (SB == 2) {
        const half2 sb2 = u2h(lds32(rp + V * 512 + 32 + g * 4));
        sg_b = __low2half2(sb2);
        sg8_b = __high2half2(sb2);
      }
      const uint4 x0 = xrow[(2 * kb) * 4];
      const uint4 x1 = xrow[(2 * kb + 1) * 4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        uint32_t a0, a1, a2, a3;
        decode_step<BITS>(cur, s, s >= 2 ? sg_b : sg_a, s >= 2 ? sg8_b : sg8_a, a0, a1, a2, a3);
        const uint4& X = (s >> 1) ? x1 : x0;
        mma16816((s & 1) ? acc2 : acc, a0, a1, a2, a3, (s & 1) ? X.z : X.x, (s & 1) ? X.w : X.y);
      }
    }
    if (t == 0) {   // column 0 is the row; the padding columns repeat it
      s_cf.part[j][g] = fadd(acc[0], acc2[0]);
      s_cf.part[j][g + 8] = fadd(acc[2], acc2[2]);
    }
  }
  for (; released < cbase + static_cast<uint32_t>(pl.n_chunks); ++released) {
    __syncwarp();
    if (lane == 0) mbar_arrive_local(&s_cf.empty[released % kCfSlots]);
  }
}

// Folded (row g, row g + 8) sums of local tile tl in the standalone GEMV's
// order: split s = vy * ksw + kw; the ksw warp partials of a CTA column vy
// in order, then, when ksg > 1, the column sums in order starting from 0.
ALM_DEV void cf_tile_sums(const QTile& w, const CfPlan& pl, int tl, int g, float& lo, float& hi) {
  const float* base = &s_cf.part[tl * pl.S][0];
  float tlo = 0.f, thi = 0.f;
  for (int vy = 0; vy < w.ksg; ++vy) {
    const float* q = base + static_cast<size_t>(vy * w.ksw) * 16;
    float clo = q[g], chi = q[g + 8];
    for (int kw = 1; kw < w.ksw; ++kw) {
      clo = fadd(clo, q[kw * 16 + g]);
      chi = fadd(chi, q[kw * 16 + g + 8]);
    }
    if (w.ksg > 1) {
      tlo = fadd(tlo, clo);
      thi = fadd(thi, chi);
    } else {
      tlo = clo;
      thi = chi;
    }
  }
  lo = tlo;
  hi = thi;
}

// Epilogues, one thread per (tile, g) pair of rows g / g + 8 (eight
// consecutive lanes per tile); the same formulas as gemv_body.cuh.
template <int EPI>
ALM_DEV void cf_epilogue(const QTile& w, const CfPlan& pl, const Epi& epi, const FwdParams& P) {
  const int n_pairs = (pl.t1 - pl.t0) * 8;
  const int pos0 = *P.io.pos;
  for (int base = 0; base < n_pairs; base += kCfConsThreads) {
    const int e = base + static_cast<int>(threadIdx.x);
    const bool live = e < n_pairs;
    const int tl = live ? e / 8 : 0, g = e % 8;
    const int tile = pl.t0 + tl;
    float lo = 0.f, hi = 0.f;
    if (live) cf_tile_sums(w, pl, tl, g, lo, hi);
    if constexpr (EPI == EPI_QKV) {
      if (!live) continue;
      const int hd = epi.head_dim, half_d = hd / 2, tph = hd / 16;
      const int tq = epi.heads * tph, tk = epi.kv_heads * tph;
      const int pos = pos0;
      if (tile < tq + tk) {
        const bool is_q = tile < tq;
        const int head = is_q ? tile / tph : (tile - tq) / tph;
        const int dlo = (tile % tph) * 8 + g, dhi = dlo + half_d;
        const size_t rb = static_cast<size_t>(pos) * hd;
        const float c = __half2float(__ldg(epi.rope + rb + dlo));
        const float sv = __half2float(__ldg(epi.rope + rb + half_d + dlo));
        const float a = round_h(lo), b = round_h(hi);
        const float rlo = fsub(fmul(a, c), fmul(b, sv));
        const float rhi = fadd(fmul(a, sv), fmul(b, c));
        if (is_q) {
          float* q = epi.q + head * hd;
          q[dlo] = rlo;
          q[dhi] = rhi;
        } else {
          const int page = epi.page_table[pos / epi.page_size];
          half* kp = epi.kcache +
                     ((static_cast<size_t>(page) * epi.kv_heads + head) * epi.page_size + pos % epi.page_size) * hd;
          kp[dlo] = __float2half_rn(rlo);
          kp[dhi] = __float2half_rn(rhi);
        }
      } else {
        const int vt = tile - tq - tk;
        const int head = vt / tph, d0 = (vt % tph) * 16 + g;
        const int page = epi.page_table[pos / epi.page_size];
        half* vp = epi.vcache +
                   ((static_cast<size_t>(page) * epi.kv_heads + head) * epi.page_size + pos % epi.page_size) * hd;
        vp[d0] = __float2half_rn(lo);
        vp[d0 + 8] = __float2half_rn(hi);
      }
    } else if constexpr (EPI == EPI_RESID) {
      // every lane takes part in the tile's sum-of-squares shuffles
      const ActIn& rs = epi.res;
      float sq = 0.f;
      const float vals[2] = {lo, hi};
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = tile * 16 + g + 8 * r;
        if (live && row < epi.n_out) {
          const float rvv = __half2float(__ldcg(rs.x + row));
          const float rw = rs.ss ? __half2float(__ldg(rs.w + row)) : 1.f;
          const float res = rs.ss ? norm_value(rvv, s_cf.den_res, rw) : rvv;
          const half s16 = __float2half_rn(fadd(res, round_h(vals[r])));
          epi.out[row] = s16;
          const float sf = __half2float(s16);
          sq = r == 0 ? fmul(sf, sf) : fadd(sq, fmul(sf, sf));
        }
      }
      sq = fadd(sq, __shfl_xor_sync(0xffffffffu, sq, 1));
      sq = fadd(sq, __shfl_xor_sync(0xffffffffu, sq, 2));
      sq = fadd(sq, __shfl_xor_sync(0xffffffffu, sq, 4));
      if (live && g == 0) epi.ss_out[tile] = sq;
    } else if constexpr (EPI == EPI_SWIGLU) {
      const int col = tile * 8 + g;
      if (live && col < epi.n_out) {
        const float gv = round_h(lo);
        const float uv = round_h(hi);
        const float sig = fdiv(1.f, fadd(1.f, expf(-gv)));
        epi.out[col] = __float2half_rn(fmul(fmul(gv, sig), uv));
      }
    }
  }
}

template <int BITS, int SB, int EPI>
ALM_DEV void cf_gemv_t(const QTile& w, const ActIn& in, const Epi& epi, uint32_t& cbase, uint32_t& n_sync,
                       const FwdParams& P, int cta) {
  const CfPlan pl = cf_plan(w, cta);
  // row denominators of deferred norms
  if (threadIdx.x < kWarp) {
    if (in.ss) {
      const float d = row_denominator(in, 0);
      if (threadIdx.x == 0) s_cf.den_in = d;
    }
  } else if (threadIdx.x < 2 * kWarp) {
    if constexpr (EPI == EPI_RESID) {
      if (epi.res.ss) {
        const float d = row_denominator(epi.res, 0);
        if (threadIdx.x == kWarp) s_cf.den_res = d;
      }
    }
  }
  cons_sync();
  if (threadIdx.x == 0) cf_mark(P, 1);
  uint4* xs = reinterpret_cast<uint4*>(cf_work());
  cf_stage(w, in, xs);
  cons_sync();
  if (threadIdx.x == 0) cf_mark(P, 2);
  cf_items<BITS, SB>(w, pl, cbase, xs, P);
  if (threadIdx.x == 0) cf_mark(P, 3);
  cbase += static_cast<uint32_t>(pl.n_chunks);
  cons_sync();
  if (threadIdx.x == 0) cf_mark(P, 4);
  cf_epilogue<EPI>(w, pl, epi, P);
  if (threadIdx.x == 0) cf_mark(P, 5);
  cf_sync(n_sync, P);
}

template <int EPI>
ALM_DEV void cf_gemv(const QTile& w, const ActIn& in, const Epi& epi, uint32_t& cbase, uint32_t& n_sync,
                     const FwdParams& P, int cta) {
  if (w.bits == 4) {
    if (w.sb == 2) cf_gemv_t<4, 2, EPI>(w, in, epi, cbase, n_sync, P, cta);
    else cf_gemv_t<4, 1, EPI>(w, in, epi, cbase, n_sync, P, cta);
  } else if (w.bits == 8) {
    if (w.sb == 2) cf_gemv_t<8, 2, EPI>(w, in, epi, cbase, n_sync, P, cta);
    else cf_gemv_t<8, 1, EPI>(w, in, epi, cbase, n_sync, P, cta);
  } else {
    cf_gemv_t<16, 0, EPI>(w, in, epi, cbase, n_sync, P, cta);
  }
}

ALM_DEV ActIn cf_raw(const half* x, int ld, int H) {
  ActIn a;
  a.x = x;
  a.ld = ld;
  a.H = H;
  set_vec(a);
  return a;
}
ALM_DEV ActIn cf_deferred(const FwdParams& P, const half* s, const float* ss, const half* w) {
  ActIn a;
  a.x = s;
  a.ld = P.hidden;
  a.ss = ss;
  a.n_ss = (P.hidden + 15) / 16;
  a.w = w;
  a.eps = P.eps;
  a.H = P.hidden;
  set_vec(a);
  return a;
}
ALM_DEV ActIn cf_layer_input(const FwdParams& P, int li) {
  return li == 0 ? cf_raw(P.embed.out, P.hidden, P.hidden)
                 : cf_deferred(P, P.s2, P.ss2, P.layers[li - 1].n_post);
}

ALM_DEV AttnArgs cf_attn_args(const FwdParams& P, int li) {
  AttnArgs a;
  const int qdim = P.heads * P.head_dim;
  a.q = P.q;
  a.ldq = qdim;
  a.kcache = P.kcache + static_cast<size_t>(li) * P.kv_layer_elems;
  a.vcache = P.vcache + static_cast<size_t>(li) * P.kv_layer_elems;
  a.page_table = P.page_table;
  a.page_size = P.page_size;
  a.heads = P.heads;
  a.kv_heads = P.kv_heads;
  a.head_dim = P.head_dim;
  a.M = 1;
  a.pos = P.io.pos;
  a.max_ctx = P.max_ctx;
  a.scores = P.scores;
  a.score_ld = P.score_ld;
  a.stats = P.stats;
  a.ctx = P.ctx;
  a.ldc = qdim;
  return a;
}

ALM_DEV void cf_layer(const FwdParams& P, int li, uint32_t& cbase, uint32_t& n_sync, int cta) {
  const FwdLayer& L = P.layers[li];
  const int qdim = P.heads * P.head_dim;
  const ActIn x_in = cf_layer_input(P, li);
  {
    Epi e;
    e.q = P.q;
    e.ldq = qdim;
    e.kcache = P.kcache + static_cast<size_t>(li) * P.kv_layer_elems;
    e.vcache = P.vcache + static_cast<size_t>(li) * P.kv_layer_elems;
    e.page_table = P.page_table;
    e.page_size = P.page_size;
    e.heads = P.heads;
    e.kv_heads = P.kv_heads;
    e.head_dim = P.head_dim;
    e.rope = P.rope;
    cf_gemv<EPI_QKV>(L.qkv, x_in, e, cbase, n_sync, P, cta);
  }
  {
    const AttnArgs a = cf_attn_args(P, li);
    const int ncm = attn_chunks_max(a);
    const int n_rg = attn_row_groups(a);
    const int kvh = a.kv_heads;
    const int n_chunks = (*a.pos + 1 + kAttnChunk - 1) / kAttnChunk;
    const int nvb1 = n_chunks * kvh * n_rg;
    unsigned char* work = cf_work();
    for (int vb = cta; vb < nvb1; vb += kCfCtas) {
      attn_scores_pages(a, vb % n_chunks, work);
      cons_sync();
      attn_scores_body<kCfThreads != 256>(a, P.sqrt_hd, vb % n_chunks, (vb / n_chunks) % kvh,
                                          vb / (n_chunks * kvh), ncm, work, s_cf.attn);
    }
    if (threadIdx.x == 0) cf_mark(P, 7);
    cf_sync(n_sync, P);
    const int nds = a.head_dim / 16, npg = attn_pv_groups(a);
    const int nvb2 = nds * kvh * npg;
    for (int vb = cta; vb < nvb2; vb += kCfCtas) {
      attn_pv_pages(a, work);
      cons_sync();
      attn_pv_body<kCfThreads != 256>(a, ncm, vb % nds, (vb / nds) % kvh, vb / (nds * kvh), work,
                                      s_cf.attn);
    }
    if (threadIdx.x == 0) cf_mark(P, 8);
    cf_sync(n_sync, P);
  }
  const ActIn n1 = cf_deferred(P, P.s1, P.ss1, L.n_in);
  {
    Epi e;
    e.out = P.s1;
    e.ldo = P.hidden;
    e.n_out = P.hidden;
    e.res = x_in;
    e.ss_out = P.ss1;
    cf_gemv<EPI_RESID>(L.o, cf_raw(P.ctx, qdim, qdim), e, cbase, n_sync, P, cta);
  }
  {
    Epi e;
    e.out = P.h;
    e.ldo = P.inter;
    e.n_out = P.inter;
    cf_gemv<EPI_SWIGLU>(L.gu, n1, e, cbase, n_sync, P, cta);
  }
  {
    Epi e;
    e.out = P.s2;
    e.ldo = P.hidden;
    e.n_out = P.hidden;
    e.res = n1;
    e.ss_out = P.ss2;
    cf_gemv<EPI_RESID>(L.down, cf_raw(P.h, P.inter, P.inter), e, cbase, n_sync, P, cta);
  }
}

__global__ void __launch_bounds__(kCfThreads, 1) cluster_fwd_kernel(const __grid_constant__ FwdParams P) {
  const int cta = static_cast<int>(cluster_rank());
  if (threadIdx.x == 0) {
    for (int i = 0; i < kCfSlots; ++i) {
      mbar_init(&s_cf.full[i], 1);
      mbar_init(&s_cf.empty[i], kCfCons);
    }
    mbar_init(&s_cf.sync[0], kCfCtas);
    mbar_init(&s_cf.sync[1], kCfCtas);
    s_cf.broken = 0;
    s_cf_tn = 0;
    s_cf_tp = 0;
    fence_mbar_init();
  }
  // every CTA's barriers are initialised before any remote arrival
  cluster_barrier_all();
  if (threadIdx.x >= kCfConsThreads) {
    // weights do not depend on earlier kernels: stream before the dependency wait
    cf_produce(P, cta);
    __syncwarp();   // lanes 1-31 wait for the streaming lane
  } else {
    grid_dep_wait();
    uint32_t cbase = 0, n_sync = 0;
    if (cta == 0) embed_body(P.embed, 0);
    cf_sync(n_sync, P);
    for (int li = 0; li < P.n_layers; ++li) cf_layer(P, li, cbase, n_sync, cta);
    grid_dep_launch();
    __syncwarp();
  }
  // no CTA leaves while another may still arrive on its barriers
  cluster_barrier_all();
}

}  // namespace

__host__ __device__ CfPlan cluster_fwd_plan(const QTile& w, int cta) {
  CfPlan p;
  const int T = w.n_tiles;
  p.t0 = static_cast<int>(static_cast<long long>(cta) * T / kCfCtas);
  p.t1 = static_cast<int>(static_cast<long long>(cta + 1) * T / kCfCtas);
  p.S = w.ksw * w.ksg;   // the standalone GEMV's K splits
  p.kps = w.kps;
  p.rec_bytes = w.rec_u4 * 16;
  p.R = kCfSlotBytes / p.rec_bytes;
  if (p.R < 1) p.R = 1;
  p.n_items = (p.t1 - p.t0) * p.S;
  p.n_rec = (p.t1 - p.t0) * w.k_blocks;
  p.n_chunks = (p.n_rec + p.R - 1) / p.R;
  p.base = reinterpret_cast<const unsigned char*>(w.data + static_cast<size_t>(p.t0) * w.k_blocks * w.rec_u4);
  return p;
}

bool cluster_fwd_weight_ok(const QTile& w) {
  if (w.layout != kLayoutTile || w.rec_u4 * 16 > kCfSlotBytes) return false;
  if (w.bits == 16 ? w.sb != 0 : (w.sb != 1 && w.sb != 2)) return false;
  for (int cta = 0; cta < kCfCtas; ++cta) {
    const CfPlan p = cluster_fwd_plan(w, cta);
    if (p.n_items > kCfMaxItems) return false;
    // an item's records span at most kCfSlots - 2 chunks (the ring cannot stall)
    if ((p.kps + p.R - 1) / p.R + 1 > kCfSlots - 2) return false;
  }
  return true;
}

size_t cluster_fwd_smem_bytes(int max_k_blocks, int head_dim) {
  size_t work = static_cast<size_t>(max_k_blocks) * 128;
  work = work > attn_scores_smem(head_dim) ? work : attn_scores_smem(head_dim);
  work = work > attn_pv_smem() ? work : attn_pv_smem();
  return kCfRingBytes + work;
}

cudaError_t cluster_fwd_init(size_t smem_bytes, int* n_clusters) {
  static std::mutex mu;
  static size_t set_bytes[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (smem_bytes > set_bytes[dev]) {
      e = cudaFuncSetAttribute(cluster_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem_bytes));
      if (e != cudaSuccess) return e;
      e = cudaFuncSetAttribute(cluster_fwd_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
      set_bytes[dev] = smem_bytes;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCfCtas, 1, 1);
  cfg.blockDim = dim3(kCfThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCfCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaOccupancyMaxActiveClusters(n_clusters, cluster_fwd_kernel, &cfg);
}

cudaError_t launch_cluster_fwd(const FwdParams& p, size_t smem_bytes, bool pdl, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCfCtas, 1, 1);
  cfg.blockDim = dim3(kCfThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCfCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, cluster_fwd_kernel, p);
}

}  // namespace alm
