// Device bodies of GQA decode / verify attention over the paged fp16 KV cache,
// shared by the standalone kernels (attention.cu) and the persistent forward
// kernel (one virtual block per call).
//
// Follows androidllm/models/llama.py:109-118 with its rounding points:
// scores = (q_fp32 . k_fp16) / sqrt(head_dim) in fp32, softmax in fp32, the
// normalised probabilities cast to fp16, then fp16(P) . fp16(V) accumulated
// in fp32 and rounded to fp16.  Because P is rounded after normalisation, the
// softmax needs the row max and sum before any P.V work, so the work is two
// passes:
//
//   scores: grid (chunk of 64 positions, kv head, group of 16 query rows).
//           q is split into fp16 hi + lo parts so two tensor-core MMAs give
//           the fp32 dot product to ~22 bits; writes masked scores and the
//           chunk's (max, sum of exp) per row.  Warps 0-3 take 16 positions
//           of the chunk each.
//   pv:     grid (16-dim slice of head_dim, kv head, group of kPvRows rows).
//           Combines the chunk statistics into the row max / sum, forms fp16
//           P while staging it in shared memory, and runs P.V on tensor cores
//           over all positions (kPvSpan at a time).
//
// Query rows of one kv head are (token m, q head within the group) pairs; row
// (m, h) attends to positions 0 .. pos0 + m (causal over the verify rows).
// Every per-row reduction has a fixed order that does not depend on how many
// rows the pass carries.
#pragma once
#include "common.cuh"
#include "kernels.cuh"

namespace alm {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / kWarp;
constexpr int kPvVld = 24;   // V slice row stride (halves): conflict-free
constexpr int kPvPld = kPvSpan + 8;   // P row stride (halves)
// one load phase per span: V vectors and score float4s within one pass of the block
static_assert(kPvSpan * 2 <= kAttnThreads * 8 && kPvRows * kPvSpan / 4 <= kAttnThreads * 4,
              "P.V span exceeds a single load phase");
// P.V: one warp per query row for the statistics
static_assert(kPvRows <= kAttnWarps, "one warp per P.V row");
// scores: q rows and the K chunk of head_dim <= 256 in one load phase
static_assert(kAttnRows * 256 / 4 <= kAttnThreads * 4 && kAttnChunk * 256 / 8 <= kAttnThreads * 8,
              "scores staging exceeds a single load phase");

// Dynamic shared memory of each pass; both end with the page numbers of the
// positions they read (one per position at most: page_size >= 1).
__host__ __device__ inline size_t attn_scores_smem(int hd) {
  return static_cast<size_t>(2 * kAttnRows + kAttnChunk) * (hd + 8) * sizeof(half) + kAttnChunk * sizeof(int);
}
__host__ __device__ inline size_t attn_pv_smem() {
  return static_cast<size_t>(kPvSpan) * kPvVld * sizeof(half) + static_cast<size_t>(kPvRows) * kPvPld * sizeof(half) +
         static_cast<size_t>(kAttnWarps) * kWarp * 8 * sizeof(float) + (kPvSpan + 1) * sizeof(int);
}
__host__ __device__ inline int attn_row_groups(const AttnArgs& a) {
  return a.seqs ? a.n_rg : (a.M * (a.heads / a.kv_heads) + kAttnRows - 1) / kAttnRows;
}
__host__ __device__ inline int attn_pv_groups(const AttnArgs& a) {
  return a.seqs ? a.n_pg : (a.M * (a.heads / a.kv_heads) + kPvRows - 1) / kPvRows;
}
__host__ __device__ inline int attn_chunks_max(const AttnArgs& a) { return (a.max_ctx + kAttnChunk - 1) / kAttnChunk; }

struct AttnShared {
  float red[kAttnWarps][kAttnRows];
  float mx[kAttnRows];
  float pm[kPvRows], pl[kPvRows];
};

ALM_DEV void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(a));
}

// Page numbers of the positions [p_begin, p_end) -> s_pg (read from global
// memory once, so every K / V load needs one round trip, not two); ptab: the
// sequence's page table (null: the pass's).
ALM_DEV void stage_pages(const AttnArgs& a, int p_begin, int p_end, int* s_pg, const int* ptab = nullptr) {
  const int* pt = ptab ? ptab : a.page_table;
  const int pg0 = p_begin / a.page_size;
  const int n_pg = (p_end - 1) / a.page_size - pg0 + 1;
  for (int i = threadIdx.x; i < n_pg; i += kAttnThreads) s_pg[i] = __ldcg(pt + pg0 + i);
}

// The sequence a scores row group (pv = false) or P.V group (pv = true)
// belongs to: its first activation row, rows, first position, page table,
// the group's index within the sequence and the sequence's first scores row
// group.  One sequence of M rows at *a.pos when the pass has no sequences.
struct AttnSeqView {
  int m0, n_tok, pos0, local, g0;
  const int* ptab;
};
ALM_DEV AttnSeqView attn_seq_view(const AttnArgs& a, int group, bool pv) {
  AttnSeqView v{0, a.M, 0, group, 0, a.page_table};
  if (!a.seqs) {
    v.pos0 = *a.pos;
    return v;
  }
  int s = 0;
  for (int i = 1; i < a.n_seq; ++i)
    if ((pv ? a.seqs[i].p0 : a.seqs[i].g0) <= group) s = i;
  const AttnSeq q = a.seqs[s];
  v.m0 = q.m0;
  v.n_tok = q.n_tok;
  v.pos0 = q.pos0;
  v.local = group - (pv ? q.p0 : q.g0);
  v.g0 = q.g0;
  v.ptab = a.page_table + q.pt_off;
  return v;
}

// Row of position pos (pages of the staged range start at page pg0).
ALM_DEV const half* kv_row(const half* cache, const int* s_pg, int pg0, int page_size, int kv_heads, int kvh,
                           int hd, int pos) {
  const int page = s_pg[pos / page_size - pg0];
  return cache + ((static_cast<size_t>(page) * kv_heads + kvh) * page_size + pos % page_size) * hd;
}

// Page numbers a scores block may read: its chunk's span of the cache
// capacity.  The page table does not change while kernels run, so this runs
// before the block waits for the kernels that produce q and K; the caller
// synchronises the block before attn_scores_body.
ALM_DEV int* attn_scores_pg(const AttnArgs& a, unsigned char* smem_raw) {
  return reinterpret_cast<int*>(smem_raw + static_cast<size_t>(2 * kAttnRows + kAttnChunk) * (a.head_dim + 8) *
                                               sizeof(half));
}
ALM_DEV void attn_scores_pages(const AttnArgs& a, int chunk, unsigned char* smem_raw) {
  if (a.seqs) return;   // a multi-sequence pass stages its sequence's pages after the wait
  const int c0 = chunk * kAttnChunk;
  if (c0 < a.max_ctx) stage_pages(a, c0, min(c0 + kAttnChunk, a.max_ctx), attn_scores_pg(a, smem_raw));
}

// Scores of (chunk, kv head, row group); n_chunks_max = the grid's chunk count.
// Precondition: attn_scores_pages for this chunk, then a block barrier.
// wait(): the dependency wait for the q rows and the pass's new K rows; a
// chunk that ends before the pass's first position has its K rows loaded
// before it (they were written by earlier passes).  Every return passes it.
template <bool NAMED = false, class Wait = NoWait>
ALM_DEV void attn_scores_body(const AttnArgs& a, float inv_sqrt_den, int chunk, int kvh, int rg, int n_chunks_max,
                              unsigned char* smem_raw, AttnShared& sh, Wait wait = Wait{}) {
  const int hd = a.head_dim, ld = hd + 8;
  half* qhi = reinterpret_cast<half*>(smem_raw);
  half* qlo = qhi + kAttnRows * ld;
  half* ks = qlo + kAttnRows * ld;   // [64][ld]
  const int* s_pg = attn_scores_pg(a, smem_raw);

  // rg: the pass's row group (the scratch layout); lg: within its sequence
  const AttnSeqView sv = attn_seq_view(a, rg, false);
  const int pos0 = sv.pos0;
  const int n_ctx = pos0 + sv.n_tok;
  const int c0 = chunk * kAttnChunk;
  if (c0 >= n_ctx) {
    wait();
    return;
  }
  const int gq = a.heads / a.kv_heads;
  const int n_rows = sv.n_tok * gq;
  const int n_rg = attn_row_groups(a);
  const int lg = sv.local;
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  // A chunk past the position of the group's last row is masked for every
  // row of the group (the first chunks of a long prefill's early groups):
  // its scores are -inf and its statistics (-inf, 0), the values the
  // products would give, written without loading K or multiplying.
  if (lg * kAttnRows >= n_rows || c0 > pos0 + min(n_rows - 1, lg * kAttnRows + kAttnRows - 1) / gq) {
    wait();
    const size_t row0 = (static_cast<size_t>(kvh) * n_rg + rg) * kAttnRows;
    for (int i = tid; i < kAttnRows * kAttnChunk; i += kAttnThreads) {
      const int p = c0 + i % kAttnChunk;
      if (p < n_ctx) a.scores[(row0 + i / kAttnChunk) * a.score_ld + p] = kNegInf;
    }
    if (tid < kAttnRows) {
      float* st = a.stats + (((static_cast<size_t>(kvh) * n_rg + rg) * n_chunks_max + chunk) * kAttnRows + tid) * 2;
      st[0] = kNegInf;
      st[1] = 0.f;
    }
    return;
  }
  const int pg0 = c0 / a.page_size;
  if (a.seqs) {
    stage_pages(a, c0, min(c0 + kAttnChunk, n_ctx), attn_scores_pg(a, smem_raw), sv.ptab);
    body_sync_t<NAMED>();
  }

  // Q rows (-> fp16 hi/lo) and the K chunk: every load issued before any is
  // used (one round trip); hd <= 256 keeps each within one pass of the block
  const int per_row = hd / 4, n4 = kAttnRows * per_row;
  const int vec_per_row = hd / 8, nv = kAttnChunk * vec_per_row;
  float4 qv[4];
  uint4 kv8[8];
  auto load_k = [&]() {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = j * kAttnThreads + tid;
      const int p = c0 + i / vec_per_row;
      kv8[j] = make_uint4(0, 0, 0, 0);
      if (i < nv && p < n_ctx)
        kv8[j] = __ldcg(reinterpret_cast<const uint4*>(kv_row(a.kcache, s_pg, pg0, a.page_size, a.kv_heads, kvh, hd,
                                                              p)) +
                        i % vec_per_row);
    }
  };
  const bool k_early = c0 + kAttnChunk <= pos0;
  if (k_early) load_k();
  wait();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = j * kAttnThreads + tid;
    const int rl = i / per_row, d4 = i % per_row;
    const int r = lg * kAttnRows + rl;
    qv[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < n4 && r < n_rows) {
      const int m = sv.m0 + r / gq, head = kvh * gq + r % gq;
      qv[j] = __ldcg(reinterpret_cast<const float4*>(a.q + static_cast<size_t>(m) * a.ldq + head * hd) + d4);
    }
  }
  if (!k_early) load_k();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = j * kAttnThreads + tid;
    if (i >= n4) break;
    const int rl = i / per_row, d = (i % per_row) * 4;
    const float vv[4] = {qv[j].x, qv[j].y, qv[j].z, qv[j].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const half h = __float2half_rn(vv[e]);
      qhi[rl * ld + d + e] = h;
      qlo[rl * ld + d + e] = __float2half_rn(vv[e] - __half2float(h));
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int i = j * kAttnThreads + tid;
    if (i >= nv) break;
    *reinterpret_cast<uint4*>(ks + (i / vec_per_row) * ld + (i % vec_per_row) * 8) = kv8[j];
  }
  body_sync_t<NAMED>();

  // warps 0-3: positions c0 + 16 w .. c0 + 16 w + 15 (two n8 tiles); all
  // warps take part in the staging above and in the block barriers below
  constexpr int kScoreWarps = kAttnChunk / 16;
  const bool mw = warp < kScoreWarps;
  const int g = lane >> 2, t = lane & 3;
  float sc[2][4];
  float rmax[2] = {kNegInf, kNegInf};
  const size_t srow0 = (static_cast<size_t>(kvh) * n_rg + rg) * kAttnRows;
  if (mw) {
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (int kk = 0; kk < hd / 16; ++kk) {
      uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
      const int arow = lane % 16, acol = kk * 16 + (lane / 16) * 8;
      ldmatrix_x4(h0, h1, h2, h3, qhi + arow * ld + acol);
      ldmatrix_x4(l0, l1, l2, l3, qlo + arow * ld + acol);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        uint32_t b0, b1;
        const int brow = warp * 16 + nt * 8 + (lane % 8);
        const int bcol = kk * 16 + ((lane / 8) % 2) * 8;
        ldmatrix_x2(b0, b1, ks + brow * ld + bcol);
        mma16816(acc[nt], h0, h1, h2, h3, b0, b1);
        mma16816(acc[nt], l0, l1, l2, l3, b0, b1);
      }
    }
    // masked scores
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rl = g + 8 * (e >> 1);
        const int r = lg * kAttnRows + rl;
        const int p = c0 + warp * 16 + nt * 8 + 2 * t + (e & 1);
        float s = kNegInf;
        if (r < n_rows && p < n_ctx && p <= pos0 + r / gq) s = fdiv(acc[nt][e], inv_sqrt_den);
        sc[nt][e] = s;
        if (p < n_ctx) a.scores[(srow0 + rl) * a.score_ld + p] = s;
        rmax[e >> 1] = fmaxf(rmax[e >> 1], s);
      }
    // row max over the chunk
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rmax[h] = fmaxf(rmax[h], __shfl_xor_sync(0xffffffffu, rmax[h], 1));
      rmax[h] = fmaxf(rmax[h], __shfl_xor_sync(0xffffffffu, rmax[h], 2));
      if (t == 0) sh.red[warp][g + 8 * h] = rmax[h];
    }
  }
  body_sync_t<NAMED>();
  if (tid < kAttnRows) {
    float mx = kNegInf;
    for (int w2 = 0; w2 < kScoreWarps; ++w2) mx = fmaxf(mx, sh.red[w2][tid]);
    sh.mx[tid] = mx;
  }
  body_sync_t<NAMED>();
  float rsum[2] = {0.f, 0.f};
  if (mw) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mx = sh.mx[g + 8 * (e >> 1)];
        const float ex = (sc[nt][e] == kNegInf) ? 0.f : expf(sc[nt][e] - mx);
        rsum[e >> 1] = fadd(rsum[e >> 1], ex);
      }
  }
  body_sync_t<NAMED>();
  if (mw) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rsum[h] = fadd(rsum[h], __shfl_xor_sync(0xffffffffu, rsum[h], 1));
      rsum[h] = fadd(rsum[h], __shfl_xor_sync(0xffffffffu, rsum[h], 2));
      if (t == 0) sh.red[warp][g + 8 * h] = rsum[h];
    }
  }
  body_sync_t<NAMED>();
  if (tid < kAttnRows) {
    float l = 0.f;
    for (int w2 = 0; w2 < kScoreWarps; ++w2) l = fadd(l, sh.red[w2][tid]);
    float* st = a.stats + (((static_cast<size_t>(kvh) * n_rg + rg) * n_chunks_max + chunk) * kAttnRows + tid) * 2;
    st[0] = sh.mx[tid];
    st[1] = l;
  }
  body_sync_t<NAMED>();   // shared memory is reused by the caller's next block
}

// P.V for (16-dim slice, kv head, group of kPvRows query rows).  Few rows
// per block keep the exp/divide work of forming P small; the rows ride in an
// m16 tile (rows >= kPvRows are zero) so the product still runs on tensor
// cores.
ALM_DEV int* attn_pv_pg(unsigned char* smem_raw) {
  return reinterpret_cast<int*>(smem_raw + static_cast<size_t>(kPvSpan) * kPvVld * sizeof(half) +
                                static_cast<size_t>(kPvRows) * kPvPld * sizeof(half) +
                                static_cast<size_t>(kAttnWarps) * kWarp * 8 * sizeof(float));
}
// Page numbers of the first positions a P.V block may read: split span sp
// (n_split > 1), else the first kPvSpan positions (before the block waits
// for the scores pass; the caller synchronises the block).
ALM_DEV void attn_pv_pages(const AttnArgs& a, unsigned char* smem_raw, int sp = 0, int n_split = 1) {
  if (a.seqs) return;   // a multi-sequence pass stages its sequence's pages after the wait
  const int b = n_split > 1 ? sp * kPvSplit : 0;
  const int e = n_split > 1 ? b + kPvSplit : kPvSpan;
  if (b < a.max_ctx) stage_pages(a, b, min(e, a.max_ctx), attn_pv_pg(smem_raw));
}

// Span split of the standalone kernel: block sp of n_split takes positions
// [sp * kPvSplit, (sp + 1) * kPvSplit) when the pass's context is longer than
// one such span (else block 0 walks every position); its fp32 partial goes to
// a.pv_part and the last block of the (slice, kv head, group) to finish adds
// the partials in span order.  A context of one span takes the unsplit path
// in block 0 (the other blocks return), so results do not depend on n_split.
// Rows whose context ends before a span get exact zeros from it, so every
// row's sum equals the one its own context length gives.
// Without SPLIT the body is compiled for one span (sp = 0, n_split = 1):
// the split's bookkeeping costs a short context about a microsecond.
// Precondition: attn_pv_pages(sp), then a block barrier.
// wait(): the dependency wait for the scores and statistics; the first
// span's V rows (written by the pass's QKV kernel and earlier passes) are
// loaded before it.  Every return passes it.
template <bool NAMED = false, bool SPLIT = false, class Wait = NoWait>
ALM_DEV void attn_pv_body(const AttnArgs& a, int n_chunks_max, int ds, int kvh, int grp, unsigned char* smem_raw,
                          AttnShared& sh, int sp = 0, int n_split = 1, Wait wait = Wait{}) {
  half* vs = reinterpret_cast<half*>(smem_raw);      // [kPvSpan][kPvVld]
  half* ps = vs + kPvSpan * kPvVld;                  // [kPvRows][kPvPld]
  float* s_acc = reinterpret_cast<float*>(ps + kPvRows * kPvPld);   // [kAttnWarps][kWarp][8]
  int* s_pg = attn_pv_pg(smem_raw);                  // pages of the current span

  const int hd = a.head_dim;
  // grp: the pass's P.V group; r0: this block's first row within its sequence
  const AttnSeqView seq = attn_seq_view(a, grp, true);
  const int pos0 = seq.pos0;
  const int n_ctx = pos0 + seq.n_tok;
  const int n_chunks = (n_ctx + kAttnChunk - 1) / kAttnChunk;
  const int gq = a.heads / a.kv_heads;
  const int n_rows = seq.n_tok * gq;
  const int n_rg = attn_row_groups(a);
  const int r0 = seq.local * kPvRows;
  const int needed = (n_ctx + kPvSplit - 1) / kPvSplit;
  const bool split = SPLIT && a.pv_part != nullptr && n_split > 1 && needed > 1;
  if (r0 >= n_rows || (!split && sp > 0) || (split && sp >= needed)) {
    wait();
    return;
  }
  const int span_begin = split ? sp * kPvSplit : 0;
  const int span_end = split ? min(span_begin + kPvSplit, n_ctx) : n_ctx;
  const int rg = seq.g0 + r0 / kAttnRows, rl0 = r0 % kAttnRows;   // scores / stats row group of the pass
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const size_t srow0 = (static_cast<size_t>(kvh) * n_rg + rg) * kAttnRows + rl0;
  const float* st = a.stats + ((static_cast<size_t>(kvh) * n_rg + rg) * n_chunks_max) * kAttnRows * 2;
  if (a.seqs) {   // the sequence's pages of the first span (attn_pv_pages staged nothing)
    stage_pages(a, span_begin, min(span_begin + kPvSpan, span_end), s_pg, seq.ptab);
    body_sync_t<NAMED>();
  }

  // One load phase for a span: the V slice (16 dims = two 16 B vectors per
  // position: span_pad * 2 <= kAttnThreads * 8 vectors) and this block's
  // scores (kPvRows * span_pad / 4 <= kAttnThreads * 4 float4s).
  uint4 v[8];
  float4 sv[4];
  auto load_v = [&](int base, int span_pad) {
    const int pg0 = base / a.page_size;
    const int nv = span_pad * 2;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = j * kAttnThreads + tid;
      const int p = base + (i >> 1);
      v[j] = make_uint4(0, 0, 0, 0);
      if (i < nv && p < n_ctx)
        v[j] = __ldcg(reinterpret_cast<const uint4*>(
                          kv_row(a.vcache, s_pg, pg0, a.page_size, a.kv_heads, kvh, hd, p) + ds * 16) +
                      (i & 1));
    }
  };
  auto load_scores = [&](int base, int span_pad) {
    const int per_row4 = span_pad / 4, np = kPvRows * per_row4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = j * kAttnThreads + tid;
      const int i_row = i / per_row4, p = base + (i % per_row4) * 4;
      sv[j] = make_float4(kNegInf, kNegInf, kNegInf, kNegInf);
      if (i < np && r0 + i_row < n_rows)
        sv[j] = __ldcg(reinterpret_cast<const float4*>(a.scores + (srow0 + i_row) * a.score_ld + p));
    }
  };

  // the first span's V slice before the wait; then the statistics of the
  // first 128 chunks (one warp per row) and the span's scores in one load
  // phase
  const int pad0 = (min(kPvSpan, span_end - span_begin) + 15) & ~15;
  load_v(span_begin, pad0);
  wait();
  float mc0[4], lc0[4];
  if (warp < kPvRows) {
    const int rl = rl0 + warp;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = j * 32 + lane;
      const float2 f = c < n_chunks ? __ldcg(reinterpret_cast<const float2*>(st + (c * kAttnRows + rl) * 2))
                                    : make_float2(kNegInf, 0.f);
      mc0[j] = f.x;
      lc0[j] = f.y;
    }
  }
  load_scores(span_begin, pad0);

  // row max / sum from the chunk statistics: one warp per row, lane l takes
  // chunks l, l+32, ... in order, then a butterfly (fixed order; chunks past
  // a row's last position contribute exact zeros)
  if (warp < kPvRows) {
    const int rl = rl0 + warp;
    float mc[4], lc[4];
    float mx = kNegInf;
#pragma unroll
    for (int j = 0; j < 4; ++j) mx = fmaxf(mx, mc0[j]);
    for (int base = 32 * 4; base < n_chunks; base += 32 * 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = base + j * 32 + lane;
        mc[j] = c < n_chunks ? __ldcg(st + (c * kAttnRows + rl) * 2) : kNegInf;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) mx = fmaxf(mx, mc[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float l = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (mc0[j] != kNegInf) l = fadd(l, fmul(lc0[j], expf(mc0[j] - mx)));
    for (int base = 32 * 4; base < n_chunks; base += 32 * 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = base + j * 32 + lane;
        mc[j] = c < n_chunks ? __ldcg(st + (c * kAttnRows + rl) * 2) : kNegInf;
        lc[j] = c < n_chunks ? __ldcg(st + (c * kAttnRows + rl) * 2 + 1) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (mc[j] != kNegInf) l = fadd(l, fmul(lc[j], expf(mc[j] - mx)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l = fadd(l, __shfl_xor_sync(0xffffffffu, l, o));
    if (lane == 0) {
      sh.pm[warp] = mx;
      sh.pl[warp] = l;
    }
  }
  body_sync_t<NAMED>();

  const int g = lane >> 2, t = lane & 3;
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  for (int base = span_begin; base < span_end; base += kPvSpan) {
    const int span = min(kPvSpan, span_end - base);
    const int span_pad = (span + 15) & ~15;
    if (base > span_begin) {   // the first span was loaded with the statistics
      stage_pages(a, base, base + span, s_pg, seq.ptab);
      body_sync_t<NAMED>();
      load_v(base, span_pad);
      load_scores(base, span_pad);
    }
    const int nv = span_pad * 2, per_row4 = span_pad / 4, np = kPvRows * per_row4;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = j * kAttnThreads + tid;
      if (i >= nv) break;
      *reinterpret_cast<uint4*>(vs + (i >> 1) * kPvVld + (i & 1) * 8) = v[j];
    }
    // P = fp16(exp(s - max) / sum) for this block's rows
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = j * kAttnThreads + tid;
      if (i >= np) break;
      const int i_row = i / per_row4, pl = (i % per_row4) * 4;
      const float e4[4] = {sv[j].x, sv[j].y, sv[j].z, sv[j].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int p = base + pl + e;
        float pv = 0.f;
        if (p < n_ctx && e4[e] != kNegInf) pv = fdiv(expf(e4[e] - sh.pm[i_row]), sh.pl[i_row]);
        ps[i_row * kPvPld + pl + e] = __float2half_rn(pv);
      }
    }
    body_sync_t<NAMED>();
    for (int kk = warp; kk < span_pad / 16; kk += kAttnWarps) {
      // A: rows g < kPvRows hold P, rows g+8 and g >= kPvRows are zero
      uint32_t a0 = 0, a2 = 0;
      if (g < kPvRows) {
        a0 = *reinterpret_cast<const uint32_t*>(ps + g * kPvPld + kk * 16 + 2 * t);
        a2 = *reinterpret_cast<const uint32_t*>(ps + g * kPvPld + kk * 16 + 8 + 2 * t);
      }
      uint32_t b0, b1, b2, b3;
      // matrices: (k0-7, n0-7) (k8-15, n0-7) (k0-7, n8-15) (k8-15, n8-15)
      const int vrow = kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
      const int vcol = (lane / 16) * 8;
      ldmatrix_x4_trans(b0, b1, b2, b3, vs + vrow * kPvVld + vcol);
      mma16816(acc[0], a0, 0u, a2, 0u, b0, b1);
      mma16816(acc[1], a0, 0u, a2, 0u, b2, b3);
    }
    body_sync_t<NAMED>();
  }

#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) s_acc[(warp * kWarp + lane) * 8 + nt * 4 + e] = acc[nt][e];
  body_sync_t<NAMED>();
  grid_dep_launch();
  const int n_pg = attn_pv_groups(a), nds = hd / 16;
  const size_t key = (static_cast<size_t>(kvh) * nds + ds) * n_pg + grp;   // (kv head, slice, group)
  float* part = split ? a.pv_part + (key * n_split + sp) * (kPvRows * 16) : nullptr;
  if (warp == 0 && g < kPvRows) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {       // rows g only (d2, d3 belong to zero rows g+8)
        float v = s_acc[lane * 8 + nt * 4 + e];
        for (int w2 = 1; w2 < kAttnWarps; ++w2) v = fadd(v, s_acc[(w2 * kWarp + lane) * 8 + nt * 4 + e]);
        const int dl = nt * 8 + 2 * t + e;
        if (split) {
          part[g * 16 + dl] = v;
          continue;
        }
        const int r = r0 + g;
        if (r < n_rows) {
          const int m = seq.m0 + r / gq, head = kvh * gq + r % gq;
          a.ctx[static_cast<size_t>(m) * a.ldc + head * hd + ds * 16 + dl] = __float2half_rn(v);
        }
      }
  }
  if (split) {
    // the last block of this (slice, kv head, group) adds the spans in order
    __threadfence();
    body_sync_t<NAMED>();
    if (tid == 0) sh.pm[0] = __int_as_float(atomicAdd(&a.pv_ticket[key], 1u) == static_cast<unsigned>(needed - 1));
    body_sync_t<NAMED>();
    if (__float_as_int(sh.pm[0]) != 0) {
      __threadfence();
      if (tid < kPvRows * 16) {
        const int rl = tid / 16, dl = tid % 16;
        const float* base = a.pv_part + key * n_split * (kPvRows * 16) + tid;
        float v = __ldcg(base);
        for (int s2 = 1; s2 < needed; ++s2) v = fadd(v, __ldcg(base + static_cast<size_t>(s2) * (kPvRows * 16)));
        const int r = r0 + rl;
        if (r < n_rows) {
          const int m = seq.m0 + r / gq, head = kvh * gq + r % gq;
          a.ctx[static_cast<size_t>(m) * a.ldc + head * hd + ds * 16 + dl] = __float2half_rn(v);
        }
      }
      if (tid == 0) atomicExch(&a.pv_ticket[key], 0u);
    }
  }
  body_sync_t<NAMED>();   // shared memory is reused by the caller's next block
}

}  // namespace alm
