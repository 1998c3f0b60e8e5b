// Single-row decode attention in one kernel: one block per kv head computes
// the scores of its query heads over the whole context, the softmax
// statistics and P.V, so a decode step launches one attention kernel instead
// of two and keeps the statistics in shared memory.  Opt-in
// (ALM_ATTN_DECODE=1): measured on B200 at the Qwen2.5-0.5B draft shape
// (2 kv heads, 640 positions) one launch takes 39.7 us against about 20 us
// for the two passes, because two blocks walk the context tile by tile at L2
// latency.
//
// Every value is computed with the arithmetic of the two-pass kernels
// (attn_body.cuh), so the results are bit-identical to them and a decode row
// equals the same row inside a multi-row verify pass:
//   * scores: q split into fp16 hi + lo, two m16n8k16 MMAs per k16 step over
//     head_dim, divided by sqrt(head_dim), masked past the row's position;
//   * per 64-position chunk: the row max over the chunk's four 16-position
//     groups, then the sum of exp(s - max) per group lane as the scores pass
//     forms it, the groups added in order;
//   * per row: the chunk statistics combined exactly as the P.V pass does
//     (lane l takes chunks l, l + 32, ..., then a butterfly);
//   * P = fp16(exp(s - max) / sum); P.V on tensor cores with k16 step i of
//     the context in warp i % 8, the warps' sums added in order per span of
//     kPvSplit positions, the spans added in order (the split P.V pass's
//     combine), then fp16.
// K and V stream through a double-buffered tile of 128 positions with
// cp.async (zero fill past the context); scores pass through the global
// scores buffer (L2), read back by the same block.
#include "attn_body.cuh"

namespace alm {
namespace {

constexpr int kDecTile = 128;                     // positions per tile (8 groups of 16)
constexpr int kDecWarps = kAttnThreads / kWarp;   // 8

ALM_DEV void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
ALM_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
ALM_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

struct DecLayout {
  int ld;             // row stride of q / K / V tiles (halves)
  size_t q_off, kv_off, acc_off, p_off, pg_off, st_off, total;
};

__host__ __device__ inline DecLayout dec_layout(int hd, int max_ctx, int page_size) {
  DecLayout L;
  L.ld = hd + 8;
  L.q_off = 0;                                                                   // qhi, qlo [16][ld]
  L.kv_off = L.q_off + static_cast<size_t>(2 * kAttnRows) * L.ld * 2;            // 2 x [128][ld]
  L.acc_off = L.kv_off + static_cast<size_t>(2 * kDecTile) * L.ld * 2;          // warp sums [warp][lane][hd / 2]
  L.p_off = L.acc_off + static_cast<size_t>(kDecWarps) * kWarp * (hd / 2) * 4;   // P [16][128 + 8]
  L.pg_off = L.p_off + static_cast<size_t>(kAttnRows) * (kDecTile + 8) * 2;      // page numbers
  const int n_pg = (max_ctx + page_size - 1) / page_size + 1;
  L.st_off = (L.pg_off + static_cast<size_t>(n_pg) * 4 + 15) / 16 * 16;          // chunk (max, sum) [chunks][16]
  const int n_chunks = (max_ctx + kAttnChunk - 1) / kAttnChunk + 2;
  L.total = L.st_off + static_cast<size_t>(n_chunks) * kAttnRows * 2 * 4;
  return L;
}

struct DecShared {
  float red[kDecWarps][kAttnRows];
  float cmx[2][kAttnRows];   // the max of the two chunks of a scores tile
  float pm[kAttnRows], pl[kAttnRows];
};

// Issue the cp.async copies of one K or V tile of kv head kvh.
ALM_DEV void dec_load_tile(const AttnArgs& a, const half* cache, int kvh, int t0, int n_ctx, const int* s_pg,
                           half* dst, int ld) {
  const int hd = a.head_dim, vpr = hd / 8;
  for (int i = threadIdx.x; i < kDecTile * vpr; i += kAttnThreads) {
    const int r = i / vpr, c = i % vpr;
    const int p = t0 + r;
    const bool ok = p < n_ctx;
    const half* src = ok ? kv_row(cache, s_pg, 0, a.page_size, a.kv_heads, kvh, hd, p) + c * 8 : cache;
    cp_async16(dst + r * ld + c * 8, src, ok);
  }
}

template <int NSL>   // head_dim / 16
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(AttnArgs a, float den) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ DecShared sh;
  const int hd = a.head_dim, kvh = blockIdx.x;
  const DecLayout L = dec_layout(hd, a.max_ctx, a.page_size);
  const int ld = L.ld;
  half* qhi = reinterpret_cast<half*>(smem_raw + L.q_off);
  half* qlo = qhi + kAttnRows * ld;
  half* kv = reinterpret_cast<half*>(smem_raw + L.kv_off);
  half* ps = reinterpret_cast<half*>(smem_raw + L.p_off);
  int* s_pg = reinterpret_cast<int*>(smem_raw + L.pg_off);
  float* st = reinterpret_cast<float*>(smem_raw + L.st_off);
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const int g = lane >> 2, t = lane & 3;

  // the page table does not change while kernels run: stage it before the wait
  stage_pages(a, 0, a.max_ctx, s_pg);
  grid_dep_wait();
  const int pos0 = *a.pos;
  const int n_ctx = pos0 + 1;
  const int gq = a.heads / a.kv_heads;
  const int n_tiles = (n_ctx + kDecTile - 1) / kDecTile;
  const int n_chunks = (n_ctx + kAttnChunk - 1) / kAttnChunk;
  const size_t srow0 = static_cast<size_t>(kvh) * kAttnRows;   // one row group of 16
  body_sync();
  dec_load_tile(a, a.kcache, kvh, 0, n_ctx, s_pg, kv, ld);
  cp_async_commit();
  // q rows -> fp16 hi / lo (rows past the group are zero)
  for (int i = tid; i < kAttnRows * hd; i += kAttnThreads) {
    const int r = i / hd, d = i % hd;
    const float v = r < gq ? __ldcg(a.q + static_cast<size_t>(kvh * gq + r) * hd + d) : 0.f;
    const half h = __float2half_rn(v);
    qhi[r * ld + d] = h;
    qlo[r * ld + d] = __float2half_rn(v - __half2float(h));
  }

  // ---- scores and chunk statistics, 128 positions (two chunks) a tile --------
  for (int it = 0; it < n_tiles; ++it) {
    const int t0 = it * kDecTile;
    if (it + 1 < n_tiles)
      dec_load_tile(a, a.kcache, kvh, t0 + kDecTile, n_ctx, s_pg, kv + ((it + 1) & 1) * kDecTile * ld, ld);
    cp_async_commit();
    cp_async_wait<1>();
    body_sync();
    const half* ks = kv + (it & 1) * kDecTile * ld;
    // warp w: positions t0 + 16 w .. + 15, the group (w % 4) of chunk 2 it + w / 4
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
    float sc[2][4];
    float rmax[2] = {kNegInf, kNegInf};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rl = g + 8 * (e >> 1);
        const int p = t0 + warp * 16 + nt * 8 + 2 * t + (e & 1);
        float s = kNegInf;
        if (rl < gq && p < n_ctx && p <= pos0) s = fdiv(acc[nt][e], den);
        sc[nt][e] = s;
        if (p < n_ctx) a.scores[(srow0 + rl) * a.score_ld + p] = s;
        rmax[e >> 1] = fmaxf(rmax[e >> 1], s);
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rmax[h] = fmaxf(rmax[h], __shfl_xor_sync(0xffffffffu, rmax[h], 1));
      rmax[h] = fmaxf(rmax[h], __shfl_xor_sync(0xffffffffu, rmax[h], 2));
      if (t == 0) sh.red[warp][g + 8 * h] = rmax[h];
    }
    body_sync();
    if (tid < 2 * kAttnRows) {   // the max of each chunk of the tile over its four groups
      const int half_t = tid / kAttnRows, row = tid % kAttnRows;
      float mx = kNegInf;
      for (int w2 = 0; w2 < 4; ++w2) mx = fmaxf(mx, sh.red[half_t * 4 + w2][row]);
      sh.cmx[half_t][row] = mx;
    }
    body_sync();
    float rsum[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mx = sh.cmx[warp / 4][g + 8 * (e >> 1)];
        const float ex = (sc[nt][e] == kNegInf) ? 0.f : expf(sc[nt][e] - mx);
        rsum[e >> 1] = fadd(rsum[e >> 1], ex);
      }
    body_sync();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rsum[h] = fadd(rsum[h], __shfl_xor_sync(0xffffffffu, rsum[h], 1));
      rsum[h] = fadd(rsum[h], __shfl_xor_sync(0xffffffffu, rsum[h], 2));
      if (t == 0) sh.red[warp][g + 8 * h] = rsum[h];
    }
    body_sync();
    if (tid < 2 * kAttnRows) {
      const int half_t = tid / kAttnRows, row = tid % kAttnRows;
      const int chunk = 2 * it + half_t;
      if (chunk * kAttnChunk < n_ctx) {
        float l = 0.f;
        for (int w2 = 0; w2 < 4; ++w2) l = fadd(l, sh.red[half_t * 4 + w2][row]);
        st[(chunk * kAttnRows + row) * 2] = sh.cmx[half_t][row];
        st[(chunk * kAttnRows + row) * 2 + 1] = l;
      }
    }
    body_sync();   // the next copy overwrites this tile's buffer
  }

  // ---- per-row statistics: the P.V pass's combine, one warp per row -----------
  dec_load_tile(a, a.vcache, kvh, 0, n_ctx, s_pg, kv, ld);
  cp_async_commit();
  for (int row = warp; row < gq; row += kDecWarps) {
    float mx = kNegInf;
    for (int base = 0; base < n_chunks; base += 32 * 4)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = base + j * 32 + lane;
        mx = fmaxf(mx, c < n_chunks ? st[(c * kAttnRows + row) * 2] : kNegInf);
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float l = 0.f;
    for (int base = 0; base < n_chunks; base += 32 * 4)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = base + j * 32 + lane;
        const float mc = c < n_chunks ? st[(c * kAttnRows + row) * 2] : kNegInf;
        const float lc = c < n_chunks ? st[(c * kAttnRows + row) * 2 + 1] : 0.f;
        if (mc != kNegInf) l = fadd(l, fmul(lc, expf(mc - mx)));
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l = fadd(l, __shfl_xor_sync(0xffffffffu, l, o));
    if (lane == 0) {
      sh.pm[row] = mx;
      sh.pl[row] = l;
    }
  }
  body_sync();

  // ---- P.V: k16 step i of the context in warp i % 8 ---------------------------
  // Spans of kPvSplit positions are summed separately and then added in span
  // order, as the split P.V pass does for a context of several spans (one
  // span: the warp sums are the result).
  float acc[NSL][2][4];   // 16-dim slice, n8 tile, fragment
#pragma unroll
  for (int sl = 0; sl < NSL; ++sl)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[sl][nt][e] = 0.f;
  float* s_acc = reinterpret_cast<float*>(smem_raw + L.acc_off);   // [warp][lane][hd / 2]
  constexpr int kPer = NSL * 8;                  // hd / 2 fragment values per lane
  constexpr int kOwn = kPer / 8;                 // output values per thread: kWarp * kPer / 256
  float tot[kOwn];
  const int pld = kDecTile + 8;
  constexpr int kTilesPerSpan = kPvSplit / kDecTile;
  static_assert(kPvSplit % kDecTile == 0, "split spans hold whole tiles");
  for (int it = 0; it < n_tiles; ++it) {
    const int t0 = it * kDecTile;
    if (it + 1 < n_tiles)
      dec_load_tile(a, a.vcache, kvh, t0 + kDecTile, n_ctx, s_pg, kv + ((it + 1) & 1) * kDecTile * ld, ld);
    cp_async_commit();
    // P of this tile's positions for every row (rows past the group are zero)
    for (int i = tid; i < kAttnRows * kDecTile; i += kAttnThreads) {
      const int r = i / kDecTile, pl = i % kDecTile, p = t0 + pl;
      float pv = 0.f;
      if (r < gq && p < n_ctx) {
        const float s = __ldcg(a.scores + (srow0 + r) * a.score_ld + p);
        if (s != kNegInf) pv = fdiv(expf(s - sh.pm[r]), sh.pl[r]);
      }
      ps[r * pld + pl] = __float2half_rn(pv);
    }
    cp_async_wait<1>();
    body_sync();
    const half* vs = kv + (it & 1) * kDecTile * ld;
    {
      const int kl = warp;   // this warp's k16 step of the tile
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(ps + g * pld + kl * 16 + 2 * t);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(ps + (g + 8) * pld + kl * 16 + 2 * t);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(ps + g * pld + kl * 16 + 8 + 2 * t);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(ps + (g + 8) * pld + kl * 16 + 8 + 2 * t);
      const int vrow = kl * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
#pragma unroll
      for (int sl = 0; sl < NSL; ++sl) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(b0, b1, b2, b3, vs + vrow * ld + sl * 16 + (lane / 16) * 8);
        mma16816(acc[sl][0], a0, a1, a2, a3, b0, b1);
        mma16816(acc[sl][1], a0, a1, a2, a3, b2, b3);
      }
    }
    const int span = it / kTilesPerSpan;
    if ((it + 1) % kTilesPerSpan == 0 || it == n_tiles - 1) {
      // end of a span: the warp sums in warp order, added to the span total
#pragma unroll
      for (int sl = 0; sl < NSL; ++sl)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            s_acc[(warp * kWarp + lane) * kPer + sl * 8 + nt * 4 + e] = acc[sl][nt][e];
            acc[sl][nt][e] = 0.f;
          }
      body_sync();
#pragma unroll
      for (int k = 0; k < kOwn; ++k) {
        const int i = k * kAttnThreads + tid;
        const int ln = i / kPer, j = i % kPer;
        float v = s_acc[ln * kPer + j];
        for (int w2 = 1; w2 < kDecWarps; ++w2) v = fadd(v, s_acc[(w2 * kWarp + ln) * kPer + j]);
        tot[k] = span == 0 ? v : fadd(tot[k], v);
      }
    }
    body_sync();   // the next copy overwrites this tile's buffer; s_acc is reused
  }
  cp_async_wait<0>();
  grid_dep_launch();
#pragma unroll
  for (int k = 0; k < kOwn; ++k) {
    const int i = k * kAttnThreads + tid;
    const int ln = i / kPer, j = i % kPer;
    const int sl = j / 8, nt = (j / 4) % 2, e = j % 4;
    const int gg = ln >> 2, tt = ln & 3;
    const int r = gg + 8 * (e >> 1);
    if (r >= gq) continue;
    const int d = sl * 16 + nt * 8 + 2 * tt + (e & 1);
    a.ctx[static_cast<size_t>(kvh * gq + r) * hd + d] = __float2half_rn(tot[k]);
  }
}

}  // namespace

size_t attn_decode_smem(int head_dim, int max_ctx, int page_size) {
  return dec_layout(head_dim, max_ctx, page_size).total;
}

cudaError_t attn_decode_init_attrs() {
  const int v = 200 * 1024;
  const auto attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
  cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<1>, attr, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_decode_kernel<2>, attr, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_decode_kernel<4>, attr, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(attn_decode_kernel<8>, attr, v);
  return e;
}

bool attn_decode_ok(const AttnArgs& a) {
  const int nsl = a.head_dim / 16;
  return a.seqs == nullptr && a.M == 1 && a.heads % a.kv_heads == 0 && a.heads / a.kv_heads <= kAttnRows && a.head_dim % 16 == 0 &&
         (nsl == 1 || nsl == 2 || nsl == 4 || nsl == 8) &&
         attn_decode_smem(a.head_dim, a.max_ctx, a.page_size) <= 200 * 1024;
}

cudaError_t launch_attn_decode(const AttnArgs& a, bool pdl, cudaStream_t st) {
  if (!attn_decode_ok(a)) return cudaErrorInvalidValue;
  const float den = static_cast<float>(sqrt(static_cast<double>(a.head_dim)));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(a.kv_heads);
  c.blockDim = dim3(kAttnThreads);
  c.dynamicSmemBytes = attn_decode_smem(a.head_dim, a.max_ctx, a.page_size);
  c.stream = st;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  switch (a.head_dim / 16) {
    case 1: return cudaLaunchKernelEx(&c, attn_decode_kernel<1>, a, den);
    case 2: return cudaLaunchKernelEx(&c, attn_decode_kernel<2>, a, den);
    case 4: return cudaLaunchKernelEx(&c, attn_decode_kernel<4>, a, den);
    default: return cudaLaunchKernelEx(&c, attn_decode_kernel<8>, a, den);
  }
}

}  // namespace alm
