// P.V of a pass with many query rows (the batched prefill): block = (kv
// head, 16-row scores group); warp w owns the 16-dim slices w, w + 8, ...
// The context is walked in spans of 128 positions: the span's V rows
// (128 x head_dim) and the 16 rows' probabilities P = fp16(exp(s - max) /
// sum) — the two-pass scheme's probabilities, from the same scores and
// chunk statistics — are staged in shared memory and multiplied on the
// tensor cores.  V is read once per 16 rows, where the decode pass (kPvRows
// rows per block, one 16-dim slice each) reads it once per kPvRows rows and
// slice.
// Only the fp32 order of the P.V sums differs from the decode pass.  It
// serves head_dim above 128; up to 128 the prefill takes the flash kernel
// below (launch_attention_prefill picks).
#include "attn_body.cuh"

namespace alm {
namespace {

constexpr int kPfSpan = 128;             // positions per span
constexpr int kPfPld = kPfSpan + 8;      // P row stride (halves)
constexpr int kPfPgMax = kPfSpan / 16 + 2;   // pages of one span (page_size >= 16)
constexpr int kPfScores = kAttnRows * kPfSpan / kAttnThreads;   // scores per thread and span
static_assert(kAttnRows * kPfSpan % kAttnThreads == 0, "scores staging layout");

__host__ __device__ inline int pf_vld(int hd) { return hd + 8; }
// two V spans (double buffer), the P span, two spans' page numbers
__host__ __device__ inline size_t pf_pv_smem(int hd) {
  return 2 * static_cast<size_t>(kPfSpan) * pf_vld(hd) * sizeof(half) +
         static_cast<size_t>(kAttnRows) * kPfPld * sizeof(half) + 2 * static_cast<size_t>(kPfPgMax) * sizeof(int);
}

ALM_DEV void cp_async16(void* smem, const void* gmem) {
  const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
ALM_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
ALM_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Row max and sum of one scores row from its chunk statistics, in the order
// the decode P.V pass uses (lane l takes chunks l, l + 32, ...; then a
// butterfly), so P is the same fp16 value in both passes.
ALM_DEV void pf_row_stats(const float* st, int rl, int n_chunks, int lane, float& mx_out, float& l_out) {
  float mx = kNegInf;
  for (int c = lane; c < n_chunks; c += 32) mx = fmaxf(mx, __ldcg(st + (c * kAttnRows + rl) * 2));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float l = 0.f;
  for (int c = lane; c < n_chunks; c += 32) {
    const float m = __ldcg(st + (c * kAttnRows + rl) * 2);
    if (m != kNegInf) l = fadd(l, fmul(__ldcg(st + (c * kAttnRows + rl) * 2 + 1), expf(m - mx)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) l = fadd(l, __shfl_xor_sync(0xffffffffu, l, o));
  mx_out = mx;
  l_out = l;
}

// Spans are pipelined: span i + 1's V rows are copied into the other buffer
// (cp.async) and its scores loaded into registers while span i is
// multiplied.  Rows past a span's end are zero in shared memory (their P is
// zero too; zero rather than stale keeps 0 * V finite).
__global__ void __launch_bounds__(kAttnThreads) attn_pv_rows16_kernel(AttnArgs a, int n_chunks_max) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float s_m[kAttnRows], s_l[kAttnRows];
  const int kvh = blockIdx.y, rg = blockIdx.z;
  grid_dep_wait();
  const int hd = a.head_dim, tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const AttnSeqView sv = attn_seq_view(a, rg, false);
  const int n_ctx = sv.pos0 + sv.n_tok;
  const int gq = a.heads / a.kv_heads;
  const int n_rows = sv.n_tok * gq;
  const int lg = sv.local;
  if (lg * kAttnRows >= n_rows) return;
  // causal bound: positions past the group's last row are masked for all
  // of its rows (their P is exactly zero and their chunks' statistics are
  // (-inf, 0), which the sums skip), so the walk stops there
  const int n_walk = min(n_ctx, sv.pos0 + min(n_rows - 1, lg * kAttnRows + kAttnRows - 1) / gq + 1);
  const int n_chunks = (n_walk + kAttnChunk - 1) / kAttnChunk;
  const int n_spans = (n_walk + kPfSpan - 1) / kPfSpan;
  const int n_rg = attn_row_groups(a);
  const size_t key = static_cast<size_t>(kvh) * n_rg + rg;
  const float* st = a.stats + key * n_chunks_max * kAttnRows * 2;
  const size_t srow0 = key * kAttnRows;
  const int vld = pf_vld(hd), vpr = hd / 8, nds = hd / 16;
  half* vbuf = reinterpret_cast<half*>(smem_raw);   // [2][kPfSpan][vld]
  half* ps = vbuf + 2 * kPfSpan * vld;              // [kAttnRows][kPfPld]
  int* s_pg = reinterpret_cast<int*>(ps + kAttnRows * kPfPld);   // [2][kPfPgMax]

  auto stage_pg = [&](int sp) {
    const int base = sp * kPfSpan, span = min(kPfSpan, n_walk - base);
    const int pg0 = base / a.page_size, n_pg = (base + span - 1) / a.page_size - pg0 + 1;
    for (int i = tid; i < n_pg; i += kAttnThreads) s_pg[(sp & 1) * kPfPgMax + i] = __ldcg(sv.ptab + pg0 + i);
  };
  auto issue_v = [&](int sp) {
    const int base = sp * kPfSpan, span = min(kPfSpan, n_walk - base), pg0 = base / a.page_size;
    const int* pg = s_pg + (sp & 1) * kPfPgMax;
    half* dst = vbuf + (sp & 1) * kPfSpan * vld;
    for (int i = tid; i < kPfSpan * vpr; i += kAttnThreads) {
      const int pr = i / vpr, part = i % vpr;
      half* d = dst + pr * vld + part * 8;
      if (pr < span)
        cp_async16(d, kv_row(a.vcache, pg, pg0, a.page_size, a.kv_heads, kvh, hd, base + pr) + part * 8);
      else
        *reinterpret_cast<uint4*>(d) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();
  };
  float sc[kPfScores];
  auto load_scores = [&](int sp) {
    const int base = sp * kPfSpan, span = min(kPfSpan, n_walk - base);
#pragma unroll
    for (int j = 0; j < kPfScores; ++j) {
      const int i = j * kAttnThreads + tid, rl = i / kPfSpan, pc = i % kPfSpan;
      sc[j] = kNegInf;
      if (lg * kAttnRows + rl < n_rows && pc < span)
        sc[j] = __ldcg(a.scores + (srow0 + rl) * a.score_ld + base + pc);
    }
  };

  for (int rl = warp; rl < kAttnRows; rl += kAttnThreads / kWarp) {
    float mx, l;
    pf_row_stats(st, rl, n_chunks, lane, mx, l);
    if (lane == 0) {
      s_m[rl] = mx;
      s_l[rl] = l;
    }
  }
  stage_pg(0);
  __syncthreads();
  issue_v(0);
  load_scores(0);
  if (n_spans > 1) stage_pg(1);
  __syncthreads();

  const int g = lane >> 2, t = lane & 3;
  float acc[2][2][4] = {};   // up to two 16-dim slices per warp (head_dim <= 256)
  for (int sp = 0; sp < n_spans; ++sp) {
    const bool more = sp + 1 < n_spans;
    if (more) issue_v(sp + 1);
    // P = fp16(exp(s - max) / sum) of this span (masked scores are -inf)
#pragma unroll
    for (int j = 0; j < kPfScores; ++j) {
      const int i = j * kAttnThreads + tid, rl = i / kPfSpan, pc = i % kPfSpan;
      float pv = 0.f;
      if (sc[j] != kNegInf) pv = fdiv(expf(sc[j] - s_m[rl]), s_l[rl]);
      ps[rl * kPfPld + pc] = __float2half_rn(pv);
    }
    if (more) load_scores(sp + 1);
    if (more)
      cp_async_wait<1>();
    else
      cp_async_wait<0>();
    __syncthreads();   // span sp's V rows and P visible
    if (sp + 2 < n_spans) stage_pg(sp + 2);   // its buffer's last reader was issue_v(sp)
    const half* vs = vbuf + (sp & 1) * kPfSpan * vld;
    for (int j = 0; j < 2; ++j) {
      const int ds = warp + j * (kAttnThreads / kWarp);
      if (ds >= nds) break;
#pragma unroll
      for (int kk = 0; kk < kPfSpan / 16; ++kk) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        ldmatrix_x4(a0, a1, a2, a3, ps + (lane % 16) * kPfPld + kk * 16 + (lane / 16) * 8);
        const int vrow = kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
        ldmatrix_x4_trans(b0, b1, b2, b3, vs + vrow * vld + ds * 16 + (lane / 16) * 8);
        mma16816(acc[j][0], a0, a1, a2, a3, b0, b1);
        mma16816(acc[j][1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();   // before the next span's P and V overwrite these buffers
  }
  for (int j = 0; j < 2; ++j) {
    const int ds = warp + j * (kAttnThreads / kWarp);
    if (ds >= nds) break;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rl = g + 8 * (e >> 1), r = lg * kAttnRows + rl;
        if (r < n_rows) {
          const int m = sv.m0 + r / gq, head = kvh * gq + r % gq;
          a.ctx[static_cast<size_t>(m) * a.ldc + head * hd + ds * 16 + nt * 8 + 2 * t + (e & 1)] =
              __float2half_rn(acc[j][nt][e]);
        }
      }
  }
  grid_dep_launch();
}


// ---- flash attention for the prefill (head_dim <= 128) ----------------------
// One pass over the context with an online softmax.  Block = (16 query rows,
// kv head); the block streams K and V in tiles of 64 positions (cp.async,
// double-buffered) up to the last position its rows can see, and warp w
// takes positions 16 w .. 16 w + 15 of every tile, keeping its own running
// max m, sum l and fp32 output O for the 16 rows.  Per tile and warp:
// S = q.k / sqrt(d) on the tensor cores (q as fp16 hi + lo, as in the decode
// passes), causal mask, m' = max(m, max S), p = exp(S - m'), l = l exp(m -
// m') + sum p, O = O exp(m - m') + fp16(p).V, the score accumulators of the
// warp's two 8-position tiles being the P operand of one 16-position k-step.
// At the end the four warps' (m, l, O) are merged through shared memory
// (warp order) and out = fp16(O / l).  A prefill chunk is compared with the
// 16-row forwards to tolerance, so its arithmetic need not follow the
// decode passes'.
constexpr int kFpWarps = 4;
constexpr int kFpRows = 16;
constexpr int kFpTile = 16 * kFpWarps;

__host__ __device__ inline size_t fp_smem(int hd) {
  const size_t ld = hd + 8;
  const size_t tiles = (2 * kFpRows * ld + 2 * 2 * kFpTile * ld) * sizeof(half);
  const size_t merge = 2 * kFpRows * ld * sizeof(half) + static_cast<size_t>(kFpWarps) * kFpRows * hd * sizeof(float);
  return tiles > merge ? tiles : merge;
}

template <int HD>
__global__ void __launch_bounds__(kFpWarps * kWarp) attn_prefill_flash_kernel(AttnArgs a, float inv_sqrt_hd) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float s_m[kFpWarps][kFpRows], s_l[kFpWarps][kFpRows];
  constexpr int LD = HD + 8, NT = HD / 8, kThreads = kFpWarps * kWarp;
  half* qhi = reinterpret_cast<half*>(smem_raw);   // [16][LD]
  half* qlo = qhi + kFpRows * LD;
  half* kbuf = qlo + kFpRows * LD;                 // [2][kFpTile][LD]
  half* vbuf = kbuf + 2 * kFpTile * LD;            // [2][kFpTile][LD]
  float* s_o = reinterpret_cast<float*>(kbuf);     // [warps][16][HD] after the tiles
  const int kvh = blockIdx.y, tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const int g = lane >> 2, t = lane & 3;
  grid_dep_wait();
  const int gq = a.heads / a.kv_heads, n_rows = a.M * gq;
  const int pos0 = *a.pos, n_ctx = pos0 + a.M;
  const int r0 = blockIdx.x * kFpRows;
  if (r0 >= n_rows) return;
  const int p_end = pos0 + (min(n_rows, r0 + kFpRows) - 1) / gq + 1;   // positions the block's rows see
  const int n_tiles = (p_end + kFpTile - 1) / kFpTile;

  auto load_tile = [&](int j) {
    half* kd = kbuf + (j & 1) * kFpTile * LD;
    half* vd = vbuf + (j & 1) * kFpTile * LD;
    constexpr int VPR = HD / 8;
    for (int i = tid; i < kFpTile * VPR; i += kThreads) {
      const int pr = i / VPR, c8 = (i % VPR) * 8, p = j * kFpTile + pr;
      if (p < n_ctx) {
        const int page = __ldg(a.page_table + p / a.page_size);
        const size_t off = ((static_cast<size_t>(page) * a.kv_heads + kvh) * a.page_size + p % a.page_size) * HD + c8;
        cp_async16(kd + pr * LD + c8, a.kcache + off);
        cp_async16(vd + pr * LD + c8, a.vcache + off);
      } else {   // past the context: zero (P is 0 there, and 0 x V must stay finite)
        *reinterpret_cast<uint4*>(kd + pr * LD + c8) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(vd + pr * LD + c8) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
  };
  load_tile(0);
  // the block's q rows as fp16 hi / lo
  for (int i = tid; i < kFpRows * (HD / 4); i += kThreads) {
    const int rl = i / (HD / 4), d = (i % (HD / 4)) * 4, r = r0 + rl;
    float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < n_rows)
      q = __ldcg(reinterpret_cast<const float4*>(a.q + static_cast<size_t>(r / gq) * a.ldq + (kvh * gq + r % gq) * HD + d));
    const float qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const half h = __float2half_rn(qq[e]);
      qhi[rl * LD + d + e] = h;
      qlo[rl * LD + d + e] = __float2half_rn(qq[e] - __half2float(h));
    }
  }

  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
  float m_run[2] = {kNegInf, kNegInf}, l_run[2] = {0.f, 0.f};
  int row_pos[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = r0 + g + 8 * h;
    row_pos[h] = r < n_rows ? pos0 + r / gq : -1;   // -1: a padding row sees nothing
  }

  for (int j = 0; j < n_tiles; ++j) {
    if (j + 1 < n_tiles) {
      load_tile(j + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const half* ks = kbuf + (j & 1) * kFpTile * LD + warp * 16 * LD;   // this warp's 16 positions
    const half* vs = vbuf + (j & 1) * kFpTile * LD + warp * 16 * LD;
    const int pw = j * kFpTile + warp * 16;
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    if (pw < p_end) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        uint32_t h0, h1, h2, h3, l0, l1, l2, l3, b0, b1, b2, b3;
        ldmatrix_x4(h0, h1, h2, h3, qhi + (lane % 16) * LD + kk * 16 + (lane / 16) * 8);
        ldmatrix_x4(l0, l1, l2, l3, qlo + (lane % 16) * LD + kk * 16 + (lane / 16) * 8);
        ldmatrix_x4(b0, b1, b2, b3, ks + ((lane % 8) + (lane / 16) * 8) * LD + kk * 16 + ((lane / 8) % 2) * 8);
        mma16816(sc[0], h0, h1, h2, h3, b0, b1);
        mma16816(sc[0], l0, l1, l2, l3, b0, b1);
        mma16816(sc[1], h0, h1, h2, h3, b2, b3);
        mma16816(sc[1], l0, l1, l2, l3, b2, b3);
      }
      // mask, tile max, online rescale
      float tmax[2] = {kNegInf, kNegInf};
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = e >> 1, p = pw + n * 8 + 2 * t + (e & 1);
          const float v = p <= row_pos[h] ? sc[n][e] * inv_sqrt_hd : kNegInf;
          sc[n][e] = v;
          tmax[h] = fmaxf(tmax[h], v);
        }
      float alpha[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 1));
        tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 2));
        const float m_new = fmaxf(m_run[h], tmax[h]);
        alpha[h] = m_new == kNegInf ? 1.f : expf(m_run[h] - m_new);
        m_run[h] = m_new;
        l_run[h] *= alpha[h];
      }
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        o[n][0] *= alpha[0];
        o[n][1] *= alpha[0];
        o[n][2] *= alpha[1];
        o[n][3] *= alpha[1];
      }
      float p[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          p[n][e] = sc[n][e] == kNegInf ? 0.f : expf(sc[n][e] - m_run[e >> 1]);
          l_run[e >> 1] += p[n][e];
        }
      const uint32_t a0 = h2u(__floats2half2_rn(p[0][0], p[0][1]));
      const uint32_t a1 = h2u(__floats2half2_rn(p[0][2], p[0][3]));
      const uint32_t a2 = h2u(__floats2half2_rn(p[1][0], p[1][1]));
      const uint32_t a3 = h2u(__floats2half2_rn(p[1][2], p[1][3]));
      const int vrow = (lane % 8) + ((lane / 8) % 2) * 8;
#pragma unroll
      for (int ds = 0; ds < HD / 16; ++ds) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(b0, b1, b2, b3, vs + vrow * LD + ds * 16 + (lane / 16) * 8);
        mma16816(o[2 * ds], a0, a1, a2, a3, b0, b1);
        mma16816(o[2 * ds + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();   // before the next load overwrites this buffer
  }
  grid_dep_launch();

  // merge the warps' (m, l, O): per row M = max m, L = sum l exp(m - M),
  // out = sum O exp(m - M) / L, warps in order
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
    if (t == 0) {
      s_m[warp][g + 8 * h] = m_run[h];
      s_l[warp][g + 8 * h] = l_run[h];
    }
  }
  float* ow = s_o + warp * kFpRows * HD;
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) ow[(g + 8 * (e >> 1)) * HD + n * 8 + 2 * t + (e & 1)] = o[n][e];
  __syncthreads();
  for (int i = tid; i < kFpRows * HD; i += kThreads) {
    const int rl = i / HD, d = i % HD, r = r0 + rl;
    if (r >= n_rows) continue;
    float mx = kNegInf;
#pragma unroll
    for (int w = 0; w < kFpWarps; ++w) mx = fmaxf(mx, s_m[w][rl]);
    float l = 0.f, v = 0.f;
#pragma unroll
    for (int w = 0; w < kFpWarps; ++w) {
      if (s_m[w][rl] == kNegInf) continue;
      const float f = expf(s_m[w][rl] - mx);
      l += s_l[w][rl] * f;
      v += s_o[(w * kFpRows + rl) * HD + d] * f;
    }
    a.ctx[static_cast<size_t>(r / gq) * a.ldc + (kvh * gq + r % gq) * HD + d] = __float2half_rn(v / l);
  }
}

}  // namespace

cudaError_t attn_prefill_init_attrs() {
  cudaError_t e = cudaFuncSetAttribute(attn_pv_rows16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(pf_pv_smem(256)));
  const auto at = cudaFuncAttributeMaxDynamicSharedMemorySize;
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_prefill_flash_kernel<16>, at, static_cast<int>(fp_smem(16)));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_prefill_flash_kernel<32>, at, static_cast<int>(fp_smem(32)));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_prefill_flash_kernel<64>, at, static_cast<int>(fp_smem(64)));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_prefill_flash_kernel<128>, at, static_cast<int>(fp_smem(128)));
  return e;
}

bool attn_prefill_flash_ok(const AttnArgs& a) {
  const int hd = a.head_dim;
  return (hd == 16 || hd == 32 || hd == 64 || hd == 128) && a.seqs == nullptr && a.pv_part == nullptr &&
         a.kv_heads > 0 && a.heads % a.kv_heads == 0 && a.page_size >= 1;
}

cudaError_t launch_attention_prefill(const AttnArgs& a, bool pdl, cudaStream_t st) {
  if (!attn_prefill_flash_ok(a)) return attn_rows16_ok(a) ? launch_attention_rows16(a, pdl, st) : launch_attention(a, pdl, st);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t c = {};
  const int gq = a.heads / a.kv_heads;
  c.gridDim = dim3((a.M * gq + kFpRows - 1) / kFpRows, a.kv_heads, 1);
  c.blockDim = dim3(kFpWarps * kWarp);
  c.dynamicSmemBytes = fp_smem(a.head_dim);
  c.stream = st;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  const float sq = static_cast<float>(1.0 / sqrt(static_cast<double>(a.head_dim)));
  switch (a.head_dim) {
    case 16: return cudaLaunchKernelEx(&c, attn_prefill_flash_kernel<16>, a, sq);
    case 32: return cudaLaunchKernelEx(&c, attn_prefill_flash_kernel<32>, a, sq);
    case 64: return cudaLaunchKernelEx(&c, attn_prefill_flash_kernel<64>, a, sq);
    default: return cudaLaunchKernelEx(&c, attn_prefill_flash_kernel<128>, a, sq);
  }
}

bool attn_rows16_ok(const AttnArgs& a) {
  return a.head_dim % 16 == 0 && a.head_dim <= 256 && a.page_size >= 16 && a.pv_part == nullptr && a.kv_heads > 0 &&
         a.heads % a.kv_heads == 0;
}

cudaError_t launch_attention_rows16(const AttnArgs& a, bool pdl, cudaStream_t st) {
  if (!attn_rows16_ok(a)) return cudaErrorInvalidValue;
  // scores and chunk statistics: the two-pass scheme's first pass
  cudaError_t e = launch_attention_scores(a, pdl, st);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(1, a.kv_heads, attn_row_groups(a));
  c.blockDim = dim3(kAttnThreads);
  c.dynamicSmemBytes = pf_pv_smem(a.head_dim);
  c.stream = st;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&c, attn_pv_rows16_kernel, a, attn_chunks_max(a));
}

}  // namespace alm
