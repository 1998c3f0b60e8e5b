// Device body of the fused dequant-GEMV: y(M, N) = x(M, K) . W(N, K)^T with
// W in the qtile layout (int4 / int8 block-quant, or fp16), M <= 16 rows.
//
// The body runs one "virtual block" (vx, vy) of the GEMV's grid and is shared
// by the standalone gemv_kernel (one CTA per virtual block) and the
// persistent forward kernel (each CTA loops over virtual blocks, phase after
// phase), so both produce bit-identical results.
//
// Work split: a block of 8 warps covers (8 / ksw) row tiles of 16; the ksw
// warps of a tile split its K range, and `ksg` blocks split K further.  Each
// warp streams its contiguous run of (tile, k64) records from HBM into a
// ring of kSlots shared-memory slots with bulk copies (TMA engine, mbarrier
// completion), decodes them to exact fp16 weights and feeds mma.sync
// m16n8k16 with fp32 accumulation.  The activation rows are staged once per
// block in shared memory, already laid out as B fragments (deferred RMSNorm
// of the previous layer is applied while staging).  Only the M real rows are
// staged; lanes whose B column is a padding row read row M-1 instead, which
// changes only output columns that are never stored (an MMA column depends
// on its own B column alone).
//
// The ring and its mbarriers persist for the CTA's lifetime: each warp counts
// the chunks that went through its ring (`seq`), which gives every chunk its
// slot and mbarrier phase.  That lets a persistent CTA issue the first chunks
// of its next virtual block (or of the next phase) before it waits for the
// activations that block needs.
//
// Partial sums are combined in a fixed order (warp order inside a block, then
// split order across blocks by the last block to finish a column), so every
// output element is summed in the same order for any M: a verify pass of k+1
// rows produces exactly the values of k+1 single-row passes.
//
// Epilogues (fused): STORE fp16; STORE32 fp32 sums (tensor-parallel partials); QKV = fp16 round, RoPE in fp32, K/V written
// to the paged cache; RESID = fp16 residual add plus per-tile sums of
// squares for the next RMSNorm; SWIGLU on interleaved gate/up rows; LOGITS =
// fp16 logits plus per-block argmax partials.  The rounding points follow
// androidllm/models/llama.py:96-146.
#pragma once
#include "act.cuh"
#include "kernels.cuh"
#include "qtile.cuh"

namespace alm {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / kWarp;

// Weight ring: kSlots slots per warp of Pipe<BITS>::kItems records each.
constexpr int kSlots = 3;
template <int BITS>
struct Pipe { static constexpr int kItems = BITS == 4 ? 4 : BITS == 8 ? 2 : 1; };
__host__ __device__ inline int pipe_items(int bits) { return bits == 4 ? 4 : bits == 8 ? 2 : 1; }
// Largest slot of any format: int4 with 32-column blocks (4 records of 36 x 16 B).
constexpr int kMaxSlotBytes = 4 * (32 + 4) * 16;
__host__ __device__ inline int gemv_slot_bytes(const QTile& w) { return pipe_items(w.bits) * w.rec_u4 * 16; }

// Chunks of 8 activation columns staged per thread per batch (all loads of a
// batch are issued before any is used, so a batch costs one memory round trip).
constexpr int kStageBatch = 4;

// k-blocks of activations one block stages: its K range.
__host__ __device__ inline int gemv_cta_nkb(const QTile& w) {
  return w.ksw * w.kps < w.k_blocks ? w.ksw * w.kps : w.k_blocks;
}
// Activation staging: per k-block, two halves (k16 steps 0-1 and 2-3), per
// row, per t = lane % 4 one uint4 {b0, b1 of the even step, b0, b1 of the odd
// step}: 128 bytes per row and k-block.
__host__ __device__ inline size_t gemv_stage_bytes(const QTile& w, int rows) {
  return static_cast<size_t>(gemv_cta_nkb(w)) * rows * 128;
}
__host__ __device__ inline int gemv_grid_x(const QTile& w) {
  const int ntc = kGemvWarps / w.ksw;
  return (w.n_tiles + ntc - 1) / ntc;
}

// The CTA's weight rings: kGemvWarps * kSlots slots of slot_bytes, then one
// mbarrier per slot.
struct Ring {
  unsigned char* base = nullptr;
  uint64_t* bars = nullptr;
  int slot_bytes = 0;
};
__host__ __device__ inline size_t ring_bytes(int slot_bytes) {
  return static_cast<size_t>(kGemvWarps) * kSlots * slot_bytes + kGemvWarps * kSlots * sizeof(uint64_t);
}
ALM_DEV Ring ring_at(unsigned char* p, int slot_bytes) {
  Ring r;
  r.base = p;
  r.slot_bytes = slot_bytes;
  r.bars = reinterpret_cast<uint64_t*>(p + static_cast<size_t>(kGemvWarps) * kSlots * slot_bytes);
  return r;
}
// Lane 0 of every warp initialises its kSlots mbarriers (once per CTA).
ALM_DEV void ring_init(const Ring& r) {
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  if (lane == 0) {
    for (int i = 0; i < kSlots; ++i) mbar_init(&r.bars[warp * kSlots + i], 1);
    fence_mbar_init();
  }
  __syncwarp();
}

template <int NT8>
struct GemvShared {
  float red[kGemvWarps][kWarp][NT8 * 4];
  float den_in[kMaxRows];
  float den_res[kMaxRows];
  int last;
  float am_v[kGemvWarps][NT8 * 8];
  int am_i[kGemvWarps][NT8 * 8];
};

// What one warp does in one virtual block.
struct GemvPlan {
  const unsigned char* gsrc;   // its first record
  int n;                       // records (k-blocks) it streams
  int n_chunks;                // ring chunks (items records each)
  int tile, kb0, kw, tl, ntc;
  int cta_kb0, cta_nkb;
  bool tile_ok;
  int vx, vy, gx;
};

ALM_DEV GemvPlan gemv_plan(const QTile& w, int items, int vx, int vy, int gx) {
  GemvPlan p;
  const int warp = threadIdx.x / kWarp;
  p.vx = vx;
  p.vy = vy;
  p.gx = gx;
  p.ntc = kGemvWarps / w.ksw;
  p.kw = warp % w.ksw;
  p.tl = warp / w.ksw;
  p.tile = vx * p.ntc + p.tl;
  p.tile_ok = p.tile < w.n_tiles;
  const int split = vy * w.ksw + p.kw;
  p.kb0 = split * w.kps;
  const int kb1 = min(p.kb0 + w.kps, w.k_blocks);
  p.n = p.tile_ok ? max(0, kb1 - p.kb0) : 0;
  p.cta_kb0 = vy * w.ksw * w.kps;
  const int cta_kb1 = min(p.cta_kb0 + w.ksw * w.kps, w.k_blocks);
  p.cta_nkb = max(0, cta_kb1 - p.cta_kb0);
  p.gsrc = reinterpret_cast<const unsigned char*>(
      w.data + (static_cast<size_t>(p.tile_ok ? p.tile : 0) * w.k_blocks + p.kb0) * w.rec_u4);
  p.n_chunks = (p.n + items - 1) / items;
  return p;
}

// Lane 0: bulk-copy chunk c of the plan into ring slot `slot`.
ALM_DEV void ring_issue_slot(const Ring& r, const GemvPlan& p, int rec_bytes, int items, int slot, int c) {
  const int warp = threadIdx.x / kWarp;
  uint64_t* bar = &r.bars[warp * kSlots + slot];
  unsigned char* dst = r.base + static_cast<size_t>(warp * kSlots + slot) * r.slot_bytes;
  const uint32_t bytes = static_cast<uint32_t>(min(items, p.n - c * items) * rec_bytes);
  mbar_expect_tx(bar, bytes);
  bulk_g2s(dst, p.gsrc + static_cast<size_t>(c) * items * rec_bytes, bytes, bar, l2_evict_first());
}
// Lane 0: bulk-copy chunk c of the plan into the ring position seq + c.
ALM_DEV void ring_issue(const Ring& r, const GemvPlan& p, int rec_bytes, int items, uint32_t seq, int c) {
  ring_issue_slot(r, p, rec_bytes, items, static_cast<int>((seq + static_cast<uint32_t>(c)) % kSlots), c);
}

// Issue the plan's first kSlots chunks (the ring must be drained and every
// thread's earlier shared-memory accesses ordered before this call, e.g. by
// __syncthreads).  Weights do not depend on earlier kernels or phases, so
// this runs before waiting for them.
template <int BITS>
ALM_DEV void gemv_issue_first(const Ring& r, const QTile& w, const GemvPlan& p, uint32_t seq) {
  if (threadIdx.x % kWarp == 0) {
    fence_proxy_async_smem();
    const int rec_bytes = w.rec_u4 * 16;
    for (int c = 0; c < p.n_chunks && c < kSlots; ++c) ring_issue(r, p, rec_bytes, Pipe<BITS>::kItems, seq, c);
  }
  __syncwarp();
}

// The rest of the virtual block after gemv_issue_first and after the inputs
// are ready: norms, staging, the streamed main loop, reductions, epilogue.
// SB: scale sets per record (0 for fp16, 1, or 2 for 32-column blocks), so
// every offset inside a record is a compile-time constant.
// xs: activation staging (gemv_stage_bytes).  Returns the chunks that went
// through the warp's ring (the caller adds them to its seq).
// Epilogue operands that do not come from the kernel the GEMV waits for, in
// the owner threads' registers.  Under programmatic dependent launch a kernel
// starts only after every CTA of its predecessor has passed its own
// dependency wait, so the kernel before that one has completed and its
// writes are visible: the residual (written two or more kernels back), its
// norm partials, the RoPE table, the positions and the page table can be
// read before this kernel's wait.  Only the standalone kernel uses this; the
// persistent forward reads them in the epilogue.
template <int NT8>
struct GemvPre {
  float res[NT8][2][2];            // RESID: residual operand (deferred norm applied)
  float cs[NT8][2], sn[NT8][2];    // QKV: RoPE cos / sin of the owner's rows
  int page[NT8][2];                // QKV: K / V cache page of the owner's rows
};

template <int NT8, int EPI>
ALM_DEV void gemv_prefetch(const QTile& w, int M, const Epi& epi, const StepIO& io, const GemvPlan& p,
                           GemvShared<NT8>& sh, GemvPre<NT8>& pre) {
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int g = lane >> 2, t = lane & 3;
  const int tile = p.tile;
  const bool owner = p.kw == 0 && p.tile_ok;
  if constexpr (EPI == EPI_RESID) {
    const ActIn& rs = epi.res;
    if (rs.ss) {
      for (int m = warp; m < M; m += kGemvWarps) {
        const float d = row_denominator(rs, m);
        if (lane == 0) sh.den_res[m] = d;
      }
      __syncthreads();
    }
    if (owner) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = tile * 16 + g + 8 * r;
        const float rw = (rs.ss && row < epi.n_out) ? __half2float(__ldg(rs.w + row)) : 1.f;
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int m = nt * 8 + 2 * t + j;
            const bool ok = m < M && row < epi.n_out;
            const float v = ok ? __half2float(__ldcg(rs.x + static_cast<size_t>(m) * rs.ld + row)) : 0.f;
            pre.res[nt][r][j] = (rs.ss && ok) ? norm_value(v, sh.den_res[m], rw) : v;
          }
      }
    }
  } else if constexpr (EPI == EPI_QKV) {
    if (owner) {
      const int hd = epi.head_dim, half_d = hd / 2, tph = hd / 16;
      const int tq = epi.heads * tph, tk = epi.kv_heads * tph;
      const int pos0 = epi.rows ? 0 : *io.pos;
      const bool rope = tile < tq + tk;
      const int dlo = (tile % tph) * 8 + g;
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int m = nt * 8 + 2 * t + j, mm = m < M ? m : 0;
          const int pos = epi.rows ? epi.rows[mm].x : pos0 + mm;
          const int* pt = epi.rows ? epi.page_table + epi.rows[mm].y : epi.page_table;
          pre.cs[nt][j] = rope ? __half2float(__ldg(epi.rope + static_cast<size_t>(pos) * hd + dlo)) : 0.f;
          pre.sn[nt][j] = rope ? __half2float(__ldg(epi.rope + static_cast<size_t>(pos) * hd + half_d + dlo)) : 0.f;
          pre.page[nt][j] = tile >= tq ? __ldg(pt + pos / epi.page_size) : 0;
        }
    }
  }
}

template <int BITS, int SB, int NT8, int EPI, bool PRE = false>
ALM_DEV int gemv_run(const QTile& w, const ActIn& in, int M, const Epi& epi, const StepIO& io,
                     float* __restrict__ part, const GemvPlan& p, const Ring& ring, uint32_t seq,
                     uint4* __restrict__ xs, GemvShared<NT8>& sh, const GemvPre<NT8>* pre = nullptr) {
  constexpr int V = QTileTraits<BITS>::kVec;
  constexpr int IPS = Pipe<BITS>::kItems;
  constexpr int REC = (V * kWarp + SB * 2) * 16;   // record bytes (w.rec_u4 * 16)
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int g = lane >> 2, t = lane & 3;
  const int ksw = w.ksw, ntc = p.ntc;
  const int kw = p.kw, tl = p.tl, tile = p.tile;
  const bool tile_ok = p.tile_ok;
  const int kb0 = p.kb0, n = p.n, n_chunks = p.n_chunks;
  const int cta_kb0 = p.cta_kb0, cta_nkb = p.cta_nkb;
  const int rec_bytes = REC;
  unsigned char* wring = ring.base + static_cast<size_t>(warp) * kSlots * ring.slot_bytes;
  uint64_t* bars = ring.bars + warp * kSlots;

  // ---- row denominators of deferred norms (one warp per row) ------------------
  // computed once the first staging batch's activation loads are in flight,
  // so the norm partials and the activations cost one memory round trip
  auto denominators = [&]() {
    for (int m = warp; m < M; m += kGemvWarps) {
      if (in.ss) {
        const float d = row_denominator(in, m);
        if (lane == 0) sh.den_in[m] = d;
      }
      if constexpr (EPI == EPI_RESID && !PRE) {
        if (epi.res.ss) {
          const float d = row_denominator(epi.res, m);
          if (lane == 0) sh.den_res[m] = d;
        }
      }
    }
    __syncthreads();
  };
  bool dens_done = false;

  // ---- stage activations as B fragments ------------------------------------
  {
    uint32_t* xw = reinterpret_cast<uint32_t*>(xs);
    const int per_row = cta_nkb * 8;           // 8-column chunks per row
    const int n_stage = per_row * M;
    const bool deferred = in.ss != nullptr;
    for (int base = 0; base < n_stage; base += kGemvThreads * kStageBatch) {
      uint4 raw[kStageBatch], wv[kStageBatch];
#pragma unroll
      for (int j = 0; j < kStageBatch; ++j) {
        const int c = base + j * kGemvThreads + threadIdx.x;
        const int m = c / per_row;
        const int col0 = cta_kb0 * 64 + (c % per_row) * 8;
        const bool ok = c < n_stage;
        raw[j] = ok ? load_row8(in, m, col0, w.k_real) : make_uint4(0, 0, 0, 0);
        wv[j] = (ok && deferred) ? load_w8(in.w, col0, w.k_real, in.vec) : make_uint4(0, 0, 0, 0);
      }
      if (!dens_done) {
        denominators();
        dens_done = true;
      }
#pragma unroll
      for (int j = 0; j < kStageBatch; ++j) {
        const int c = base + j * kGemvThreads + threadIdx.x;
        if (c >= n_stage) break;
        const int m = c / per_row;
        const int rem = c % per_row;
        const int kbl = rem / 8, c8 = rem % 8;
        const int s = c8 >> 1, hi8 = c8 & 1;
        const int h = s >> 1, r = (s & 1) * 2 + hi8;
        uint32_t words[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
        if (deferred) {
          const float den = sh.den_in[m];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float a0 = norm_value(u4_half(raw[j], 2 * q), den, u4_half(wv[j], 2 * q));
            const float a1 = norm_value(u4_half(raw[j], 2 * q + 1), den, u4_half(wv[j], 2 * q + 1));
            words[q] = h2u(__floats2half2_rn(a0, a1));
          }
        }
#pragma unroll
        for (int tt = 0; tt < 4; ++tt)
          xw[((((kbl * 2 + h) * M + m) * 4 + tt) * 4) + r] = words[tt];
      }
    }
    if (!dens_done) denominators();
  }
  __syncthreads();

  // ---- main loop -------------------------------------------------------------
  // Two accumulator chains (even / odd k16 steps) so consecutive MMAs do not
  // wait on each other; they are added in a fixed order at the end.
  float acc[NT8][4], acc2[NT8][4];
#pragma unroll
  for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[nt][j] = acc2[nt][j] = 0.f;

  // B fragments of this lane: row nt * 8 + g (padding columns read row M-1),
  // 4 * M uint4 per half k-block
  const uint4* xrow[NT8];
#pragma unroll
  for (int nt = 0; nt < NT8; ++nt) xrow[nt] = xs + min(nt * 8 + g, M - 1) * 4 + t;
  const int xhalf = 4 * M;
  // one record: decode the lane's weights of a (tile, k-block) and feed 4 MMAs
  auto record = [&](const unsigned char* rp, int kbl) {
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
    uint4 xf[NT8][2];
#pragma unroll
    for (int nt = 0; nt < NT8; ++nt) {
      xf[nt][0] = xrow[nt][(2 * kbl) * xhalf];
      xf[nt][1] = xrow[nt][(2 * kbl + 1) * xhalf];
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      uint32_t a0, a1, a2, a3;
      decode_step<BITS>(cur, s, s >= 2 ? sg_b : sg_a, s >= 2 ? sg8_b : sg8_a, a0, a1, a2, a3);
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt) {
        const uint4& X = xf[nt][s >> 1];
        const uint32_t b0 = (s & 1) ? X.z : X.x;
        const uint32_t b1 = (s & 1) ? X.w : X.y;
        mma16816((s & 1) ? acc2[nt] : acc[nt], a0, a1, a2, a3, b0, b1);
      }
    }
  };
  int consumed = 0;
  bool stream_ok = true;
  int slot = static_cast<int>(seq % kSlots);
  uint32_t phase = (seq / kSlots) & 1u;
  for (int c = 0; c < n_chunks; ++c) {
    if (!mbar_wait(&bars[slot], phase)) {
      stream_ok = false;
      break;
    }
    const unsigned char* sp = wring + slot * ring.slot_bytes;
    const int kbl0 = kb0 + c * IPS - cta_kb0;
    const int cnt = min(IPS, n - c * IPS);
    if (cnt == IPS) {
#pragma unroll
      for (int j = 0; j < IPS; ++j) record(sp + j * REC, kbl0 + j);
    } else {
#pragma unroll
      for (int j = 0; j < IPS; ++j)
        if (j < cnt) record(sp + j * REC, kbl0 + j);
    }
    consumed = c + 1;
    __syncwarp();
    if (lane == 0 && c + kSlots < n_chunks) {
      fence_proxy_async_smem();   // this slot's reads are done before the copy overwrites it
      ring_issue_slot(ring, p, rec_bytes, IPS, slot, c + kSlots);
    }
    if (++slot == kSlots) {
      slot = 0;
      phase ^= 1u;
    }
  }
  int issued = n_chunks;
  if (!stream_ok) {
    // a copy never completed: report it and let every copy still in flight
    // land before the slots are used again
    if (lane == 0 && io.err) atomicExch(io.err, 2);
    issued = min(n_chunks, consumed + kSlots);
    for (int c = consumed; c < issued; ++c) {
      const uint32_t s_pos = seq + static_cast<uint32_t>(c);
      mbar_wait(&bars[s_pos % kSlots], (s_pos / kSlots) & 1u);
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[nt][j] = fadd(acc[nt][j], acc2[nt][j]);

  grid_dep_launch();

  // ---- reduce the ksw warps of a tile (fixed order) -------------------------
  if (ksw > 1) {
#pragma unroll
    for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) sh.red[warp][lane][nt * 4 + j] = acc[nt][j];
    __syncthreads();
    if (kw == 0) {
      for (int k2 = 1; k2 < ksw; ++k2)
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[nt][j] = fadd(acc[nt][j], sh.red[warp + k2][lane][nt * 4 + j]);
    }
  }

  // ---- reduce across the ksg blocks of a column (last block, fixed order) ----
  if (w.ksg > 1) {
    const size_t tiles_pad = static_cast<size_t>(p.gx) * ntc;
    if (kw == 0 && tile_ok) {
      float4* dst = reinterpret_cast<float4*>(part) +
                    ((static_cast<size_t>(p.vy) * tiles_pad + tile) * kWarp + lane) * NT8;
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt) dst[nt] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) sh.last = atomicAdd(&w.counters[p.vx], 1u) == static_cast<unsigned>(w.ksg - 1);
    __syncthreads();
    if (!sh.last) return issued;
    __threadfence();
    if (kw == 0 && tile_ok) {
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[nt][j] = 0.f;
      for (int sp = 0; sp < w.ksg; ++sp) {
        const float4* src = reinterpret_cast<const float4*>(part) +
                            ((static_cast<size_t>(sp) * tiles_pad + tile) * kWarp + lane) * NT8;
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt) {
          const float4 pv = __ldcg(src + nt);
          acc[nt][0] = fadd(acc[nt][0], pv.x);
          acc[nt][1] = fadd(acc[nt][1], pv.y);
          acc[nt][2] = fadd(acc[nt][2], pv.z);
          acc[nt][3] = fadd(acc[nt][3], pv.w);
        }
      }
    }
    if (threadIdx.x == 0) atomicExch(&w.counters[p.vx], 0u);
  }

  // ---- epilogues -------------------------------------------------------------
  const bool owner = kw == 0 && tile_ok;
  if constexpr (EPI == EPI_STORE) {
    if (owner) {
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int m = nt * 8 + 2 * t + j, row = tile * 16 + g + 8 * r;
            if (m < M && row < epi.n_out)
              epi.out[static_cast<size_t>(m) * epi.ldo + row] = __float2half_rn(acc[nt][2 * r + j]);
          }
    }
  } else if constexpr (EPI == EPI_STORE32) {
    if (owner) {
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int m = nt * 8 + 2 * t + j, row = tile * 16 + g + 8 * r;
            if (m < M && row < epi.n_out) epi.out32[static_cast<size_t>(m) * epi.ldo + row] = acc[nt][2 * r + j];
          }
    }
  } else if constexpr (EPI == EPI_QKV) {
    if (owner) {
      const int hd = epi.head_dim, half_d = hd / 2, tph = hd / 16;
      const int tq = epi.heads * tph, tk = epi.kv_heads * tph;
      // row m's position and page table: pos0 + m, or its sequence's (epi.rows)
      const int pos0 = epi.rows ? 0 : *io.pos;
      auto row_pos = [&](int m) { return epi.rows ? epi.rows[m].x : pos0 + m; };
      auto row_pages = [&](int m) { return epi.rows ? epi.page_table + epi.rows[m].y : epi.page_table; };
      if (tile < tq + tk) {
        const bool is_q = tile < tq;
        const int head = is_q ? tile / tph : (tile - tq) / tph;
        const int dlo = (tile % tph) * 8 + g, dhi = dlo + half_d;
        float cs[NT8][2], sn[NT8][2];
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            if constexpr (PRE) {
              cs[nt][j] = pre->cs[nt][j];
              sn[nt][j] = pre->sn[nt][j];
            } else {
              const int m = nt * 8 + 2 * t + j;
              const size_t rb = static_cast<size_t>(row_pos(m < M ? m : 0)) * hd;
              cs[nt][j] = __half2float(__ldg(epi.rope + rb + dlo));
              sn[nt][j] = __half2float(__ldg(epi.rope + rb + half_d + dlo));
            }
          }
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int m = nt * 8 + 2 * t + j;
            if (m >= M) continue;
            const int pos = row_pos(m);
            const float a = round_h(acc[nt][j]), b = round_h(acc[nt][2 + j]);
            const float c = cs[nt][j];
            const float sv = sn[nt][j];
            const float rlo = fsub(fmul(a, c), fmul(b, sv));
            const float rhi = fadd(fmul(a, sv), fmul(b, c));
            if (is_q) {
              float* q = epi.q + static_cast<size_t>(m) * epi.ldq + head * hd;
              q[dlo] = rlo;
              q[dhi] = rhi;
            } else {
              const int page = PRE ? pre->page[nt][j] : row_pages(m)[pos / epi.page_size];
              half* kp = epi.kcache +
                         ((static_cast<size_t>(page) * epi.kv_heads + head) * epi.page_size + pos % epi.page_size) * hd;
              kp[dlo] = __float2half_rn(rlo);
              kp[dhi] = __float2half_rn(rhi);
            }
          }
      } else {
        const int vt = tile - tq - tk;
        const int head = vt / tph, d0 = (vt % tph) * 16 + g;
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int m = nt * 8 + 2 * t + j;
            if (m >= M) continue;
            const int pos = row_pos(m);
            const int page = PRE ? pre->page[nt][j] : row_pages(m)[pos / epi.page_size];
            half* vp = epi.vcache +
                       ((static_cast<size_t>(page) * epi.kv_heads + head) * epi.page_size + pos % epi.page_size) * hd;
            vp[d0] = __float2half_rn(acc[nt][j]);
            vp[d0 + 8] = __float2half_rn(acc[nt][2 + j]);
          }
      }
    }
  } else if constexpr (EPI == EPI_RESID) {
    if (owner) {
      const ActIn& rs = epi.res;
      float rv[NT8][2][2], rw[2];
      if constexpr (!PRE) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int row = tile * 16 + g + 8 * r;
          rw[r] = (rs.ss && row < epi.n_out) ? __half2float(__ldg(rs.w + row)) : 1.f;
        }
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
          for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int m = nt * 8 + 2 * t + j, row = tile * 16 + g + 8 * r;
              const bool ok = m < M && row < epi.n_out;
              rv[nt][r][j] = ok ? __half2float(__ldcg(rs.x + static_cast<size_t>(m) * rs.ld + row)) : 0.f;
            }
      }
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int m = nt * 8 + 2 * t + j;
          float sq = 0.f;
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const int row = tile * 16 + g + 8 * r;
            if (m < M && row < epi.n_out) {
              const float o = round_h(acc[nt][2 * r + j]);
              float res;
              if constexpr (PRE)
                res = pre->res[nt][r][j];
              else
                res = rs.ss ? norm_value(rv[nt][r][j], sh.den_res[m], rw[r]) : rv[nt][r][j];
              const half s16 = __float2half_rn(fadd(res, o));
              epi.out[static_cast<size_t>(m) * epi.ldo + row] = s16;
              const float sf = __half2float(s16);
              sq = r == 0 ? fmul(sf, sf) : fadd(sq, fmul(sf, sf));
            }
          }
          sq = fadd(sq, __shfl_xor_sync(0xffffffffu, sq, 4));
          sq = fadd(sq, __shfl_xor_sync(0xffffffffu, sq, 8));
          sq = fadd(sq, __shfl_xor_sync(0xffffffffu, sq, 16));
          if (g == 0 && m < M) epi.ss_out[static_cast<size_t>(m) * w.n_tiles + tile] = sq;
        }
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    if (owner) {
      const int col = tile * 8 + g;
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int m = nt * 8 + 2 * t + j;
          if (m < M && col < epi.n_out) {
            const float gv = round_h(acc[nt][j]);
            const float uv = round_h(acc[nt][2 + j]);
            const float sig = fdiv(1.f, fadd(1.f, expf(-gv)));
            epi.out[static_cast<size_t>(m) * epi.ldo + col] = __float2half_rn(fmul(fmul(gv, sig), uv));
          }
        }
    }
  } else if constexpr (EPI == EPI_LOGITS) {
    if (kw == 0) {
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int m = nt * 8 + 2 * t + j;
          float bv = kNegInf;
          int bi = 0x7fffffff;
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const int row = tile * 16 + g + 8 * r;
            if (tile_ok && m < M && row < epi.n_out) {
              const half l16 = __float2half_rn(acc[nt][2 * r + j]);
              epi.out[static_cast<size_t>(m) * epi.ldo + row] = l16;
              const float lv = __half2float(l16);
              if (better(lv, row, bv, bi)) { bv = lv; bi = row; }
            }
          }
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
          }
          if (g == 0) {
            sh.am_v[tl][nt * 8 + 2 * t + j] = bv;
            sh.am_i[tl][nt * 8 + 2 * t + j] = bi;
          }
        }
    }
    __syncthreads();
    if (threadIdx.x < M) {
      const int m = threadIdx.x;
      float bv = kNegInf;
      int bi = 0x7fffffff;
      for (int k = 0; k < ntc; ++k)
        if (better(sh.am_v[k][m], sh.am_i[k][m], bv, bi)) { bv = sh.am_v[k][m]; bi = sh.am_i[k][m]; }
      epi.am_val[static_cast<size_t>(m) * p.gx + p.vx] = bv;
      epi.am_idx[static_cast<size_t>(m) * p.gx + p.vx] = bi;
    }
  }
  return issued;
}

}  // namespace alm
