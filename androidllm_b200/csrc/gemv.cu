// Fused dequant-GEMV for the verify path: y(M, N) = x(M, K) . W(N, K)^T with
// W in the qtile layout (int4 / int8 block-quant, or fp16), M <= 16 rows.
//
// Work split: a CTA of 8 warps covers (8 / ksw) row tiles of 16; the ksw warps
// of a tile split its K range, and `ksg` CTAs split K further.  Each warp
// streams its contiguous run of k64 blocks straight from HBM into registers
// (a rolling prefetch of U blocks), decodes them to exact fp16 weights and
// feeds mma.sync m16n8k16 with fp32 accumulation.  The activation rows are
// staged once per CTA in shared memory, already laid out as B fragments
// (deferred RMSNorm of the previous layer is applied while staging).
//
// Partial sums are combined in a fixed order (warp order inside a CTA, then
// split order across CTAs by the last CTA to finish a column), so every
// output element is summed in the same order for any M: a verify pass of k+1
// rows produces exactly the values of k+1 single-row passes.
//
// Epilogues (fused): STORE fp16; QKV = fp16 round, RoPE in fp32, K/V written
// to the paged cache; RESID = fp16 residual add plus per-tile sums of
// squares for the next RMSNorm; SWIGLU on interleaved gate/up rows; LOGITS =
// fp16 logits plus per-CTA argmax partials.  The rounding points follow
// androidllm/models/llama.py:96-146.
#include <algorithm>

#include "act.cuh"
#include "kernels.cuh"
#include "qtile.cuh"

namespace alm {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / kWarp;
constexpr size_t kGemvMaxSmem = 200 * 1024;   // dynamic shared memory limit per CTA

// Weight ring: each warp streams its contiguous run of records into
// kSlots shared-memory slots of Pipe<BITS>::kItems records each, one bulk copy
// (TMA engine) per slot, while it decodes the previous slots.
constexpr int kSlots = 3;
template <int BITS>
struct Pipe { static constexpr int kItems = BITS == 4 ? 4 : BITS == 8 ? 2 : 1; };

// Dynamic shared memory of one CTA: activation fragments, weight rings, mbarriers.
inline size_t gemv_smem_bytes(const QTile& w, int nt8, int items) {
  const int cta_nkb = w.ksw * w.kps < w.k_blocks ? w.ksw * w.kps : w.k_blocks;
  const size_t x = static_cast<size_t>(cta_nkb) * nt8 * 2 * kWarp * sizeof(uint4);
  const size_t ring = static_cast<size_t>(kWarps) * kSlots * items * w.rec_u4 * sizeof(uint4);
  return x + ring + kWarps * kSlots * sizeof(uint64_t);
}

// Chunks of 8 activation columns staged per thread per batch (all loads of a
// batch are issued before any is used, so a batch costs one memory round trip).
constexpr int kStageBatch = 4;

ALM_DEV bool better(float v1, int i1, float v2, int i2) {
  return v1 > v2 || (v1 == v2 && i1 < i2);
}

template <int BITS, int NT8, int EPI>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(QTile w, ActIn in, int M, Epi epi, StepIO io,
                                                        float* __restrict__ part) {
  extern __shared__ uint4 xs[];  // [kb_local][NT8][2][32] uint4, then weight rings, then mbarriers
  __shared__ float red[kWarps][kWarp][NT8 * 4];
  __shared__ float s_den_in[kMaxRows];
  __shared__ float s_den_res[kMaxRows];
  __shared__ int s_last;
  __shared__ float s_am_v[kWarps][NT8 * 8];
  __shared__ int s_am_i[kWarps][NT8 * 8];

  constexpr int V = QTileTraits<BITS>::kVec;
  constexpr int IPS = Pipe<BITS>::kItems;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int g = lane >> 2, t = lane & 3;
  const int ksw = w.ksw, ntc = kWarps / ksw;
  const int kw = warp % ksw, tl = warp / ksw;
  const int tile = blockIdx.x * ntc + tl;
  const bool tile_ok = tile < w.n_tiles;
  const int split = blockIdx.y * ksw + kw;
  const int kb0 = split * w.kps;
  const int kb1 = min(kb0 + w.kps, w.k_blocks);
  const int n = tile_ok ? max(0, kb1 - kb0) : 0;
  const int cta_kb0 = blockIdx.y * ksw * w.kps;
  const int cta_kb1 = min(cta_kb0 + ksw * w.kps, w.k_blocks);
  const int cta_nkb = max(0, cta_kb1 - cta_kb0);

  // ---- weight stream (does not depend on the previous kernel) -------------
  const int rec_bytes = w.rec_u4 * 16;
  const int slot_bytes = IPS * rec_bytes;
  unsigned char* ring = reinterpret_cast<unsigned char*>(xs + static_cast<size_t>(cta_nkb) * NT8 * 2 * kWarp) +
                        static_cast<size_t>(warp) * kSlots * slot_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(xs) +
                                               static_cast<size_t>(cta_nkb) * NT8 * 2 * kWarp * 16 +
                                               static_cast<size_t>(kWarps) * kSlots * slot_bytes) + warp * kSlots;
  const unsigned char* gsrc = reinterpret_cast<const unsigned char*>(
      w.data + (static_cast<size_t>(tile_ok ? tile : 0) * w.k_blocks + kb0) * w.rec_u4);
  const int n_chunks = (n + IPS - 1) / IPS;
  auto issue = [&](int c) {   // lane 0: bulk-copy chunk c into its slot
    const int slot = c % kSlots;
    const uint32_t bytes = static_cast<uint32_t>(min(IPS, n - c * IPS) * rec_bytes);
    mbar_expect_tx(&bars[slot], bytes);
    bulk_g2s(ring + slot * slot_bytes, gsrc + static_cast<size_t>(c) * slot_bytes, bytes, &bars[slot]);
  };
  if (lane == 0) {
    for (int i = 0; i < kSlots; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    for (int c = 0; c < n_chunks && c < kSlots; ++c) issue(c);
  }
  __syncwarp();

  grid_dep_wait();

  // ---- row denominators of deferred norms (one warp per row) ------------------
  for (int m = warp; m < M; m += kWarps) {
    if (in.ss) {
      const float d = row_denominator(in, m);
      if (lane == 0) s_den_in[m] = d;
    }
    if constexpr (EPI == EPI_RESID) {
      if (epi.res.ss) {
        const float d = row_denominator(epi.res, m);
        if (lane == 0) s_den_res[m] = d;
      }
    }
  }
  __syncthreads();

  // ---- stage activations as B fragments ------------------------------------
  {
    uint32_t* xw = reinterpret_cast<uint32_t*>(xs);
    const int per_row = cta_nkb * 8;           // 8-column chunks per row
    const int n_chunks = per_row * M;          // rows >= M are zeroed in registers, not staged
    const bool deferred = in.ss != nullptr;
    for (int base = 0; base < n_chunks; base += kThreads * kStageBatch) {
      uint4 raw[kStageBatch], wv[kStageBatch];
#pragma unroll
      for (int j = 0; j < kStageBatch; ++j) {
        const int c = base + j * kThreads + threadIdx.x;
        const int m = c / per_row;
        const int col0 = cta_kb0 * 64 + (c % per_row) * 8;
        const bool ok = c < n_chunks && m < M;
        raw[j] = ok ? load_row8(in, m, col0, w.k_real) : make_uint4(0, 0, 0, 0);
        wv[j] = (ok && deferred) ? load_w8(in.w, col0, w.k_real, in.vec) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < kStageBatch; ++j) {
        const int c = base + j * kThreads + threadIdx.x;
        if (c >= n_chunks) break;
        const int m = c / per_row;
        const int rem = c % per_row;
        const int kbl = rem / 8, c8 = rem % 8;
        const int s = c8 >> 1, hi8 = c8 & 1;
        const int nt = m >> 3, h = s >> 1, r = (s & 1) * 2 + hi8;
        uint32_t words[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
        if (deferred && m < M) {
          const float den = s_den_in[m];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float a0 = norm_value(u4_half(raw[j], 2 * q), den, u4_half(wv[j], 2 * q));
            const float a1 = norm_value(u4_half(raw[j], 2 * q + 1), den, u4_half(wv[j], 2 * q + 1));
            words[q] = h2u(__floats2half2_rn(a0, a1));
          }
        }
#pragma unroll
        for (int tt = 0; tt < 4; ++tt)
          xw[(((kbl * NT8 + nt) * 2 + h) * kWarp + (m & 7) * 4 + tt) * 4 + r] = words[tt];
      }
    }
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

  const bool two_sets = w.sb == 2;
  int consumed = 0;
  bool stream_ok = true;
  for (int c = 0; c < n_chunks; ++c) {
    const int slot = c % kSlots;
    if (!mbar_wait(&bars[slot], static_cast<uint32_t>((c / kSlots) & 1))) {
      stream_ok = false;
      break;
    }
    const unsigned char* sp = ring + slot * slot_bytes;
    const int cnt = min(IPS, n - c * IPS);
#pragma unroll
    for (int j = 0; j < IPS; ++j) {
      if (j < cnt) {
        const unsigned char* rp = sp + j * rec_bytes;
        uint4 cur[V];
#pragma unroll
        for (int v = 0; v < V; ++v) cur[v] = lds128(rp + v * 512 + lane * 16);
        half2 sg_a = __float2half2_rn(1.f), sg8_a = sg_a, sg_b = sg_a, sg8_b = sg_a;
        if constexpr (BITS != 16) {
          const half2 sa = u2h(lds32(rp + V * 512 + g * 4));
          const half2 sb2 = two_sets ? u2h(lds32(rp + V * 512 + 32 + g * 4)) : sa;
          sg_a = __low2half2(sa);
          sg8_a = __high2half2(sa);
          sg_b = __low2half2(sb2);
          sg8_b = __high2half2(sb2);
        }
        const int kbl = kb0 + c * IPS + j - cta_kb0;
        uint4 xf[NT8][2];
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt) {
          const bool live = nt * 8 + g < M;   // B column g of n8 tile nt is activation row nt*8+g
          xf[nt][0] = live ? xs[((kbl * NT8 + nt) * 2 + 0) * kWarp + lane] : make_uint4(0, 0, 0, 0);
          xf[nt][1] = live ? xs[((kbl * NT8 + nt) * 2 + 1) * kWarp + lane] : make_uint4(0, 0, 0, 0);
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
      }
    }
    consumed = c + 1;
    __syncwarp();
    if (lane == 0 && c + kSlots < n_chunks) {
      fence_proxy_async_smem();   // this slot's reads are done before the copy overwrites it
      issue(c + kSlots);
    }
  }
  if (!stream_ok) {
    // a copy never completed: report it and let every copy still in flight
    // land before the CTA's shared memory is released
    if (lane == 0 && io.err) atomicExch(io.err, 2);
    const int issued = min(n_chunks, consumed + kSlots);
    for (int c = consumed; c < issued; ++c) mbar_wait(&bars[c % kSlots], static_cast<uint32_t>((c / kSlots) & 1));
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
      for (int j = 0; j < 4; ++j) red[warp][lane][nt * 4 + j] = acc[nt][j];
    __syncthreads();
    if (kw == 0) {
      for (int k2 = 1; k2 < ksw; ++k2)
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[nt][j] = fadd(acc[nt][j], red[warp + k2][lane][nt * 4 + j]);
    }
  }

  // ---- reduce across the ksg CTAs of a column (last CTA, fixed order) -------
  if (w.ksg > 1) {
    const size_t tiles_pad = static_cast<size_t>(gridDim.x) * ntc;
    if (kw == 0 && tile_ok) {
      float4* dst = reinterpret_cast<float4*>(part) +
                    ((static_cast<size_t>(blockIdx.y) * tiles_pad + tile) * kWarp + lane) * NT8;
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt) dst[nt] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&w.counters[blockIdx.x], 1u) == static_cast<unsigned>(w.ksg - 1);
    __syncthreads();
    if (!s_last) return;
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
          const float4 p = __ldcg(src + nt);
          acc[nt][0] = fadd(acc[nt][0], p.x);
          acc[nt][1] = fadd(acc[nt][1], p.y);
          acc[nt][2] = fadd(acc[nt][2], p.z);
          acc[nt][3] = fadd(acc[nt][3], p.w);
        }
      }
    }
    if (threadIdx.x == 0) atomicExch(&w.counters[blockIdx.x], 0u);
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
  } else if constexpr (EPI == EPI_QKV) {
    if (owner) {
      const int hd = epi.head_dim, half_d = hd / 2, tph = hd / 16;
      const int tq = epi.heads * tph, tk = epi.kv_heads * tph;
      const int pos0 = *io.pos;
      if (tile < tq + tk) {
        const bool is_q = tile < tq;
        const int head = is_q ? tile / tph : (tile - tq) / tph;
        const int dlo = (tile % tph) * 8 + g, dhi = dlo + half_d;
        float cs[NT8][2], sn[NT8][2];
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int m = nt * 8 + 2 * t + j;
            const size_t rb = static_cast<size_t>(m < M ? pos0 + m : pos0) * hd;
            cs[nt][j] = __half2float(__ldg(epi.rope + rb + dlo));
            sn[nt][j] = __half2float(__ldg(epi.rope + rb + half_d + dlo));
          }
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int m = nt * 8 + 2 * t + j;
            if (m >= M) continue;
            const int pos = pos0 + m;
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
              const int page = epi.page_table[pos / epi.page_size];
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
            const int pos = pos0 + m;
            const int page = epi.page_table[pos / epi.page_size];
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
              const float res = rs.ss ? norm_value(rv[nt][r][j], s_den_res[m], rw[r]) : rv[nt][r][j];
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
            s_am_v[tl][nt * 8 + 2 * t + j] = bv;
            s_am_i[tl][nt * 8 + 2 * t + j] = bi;
          }
        }
    }
    __syncthreads();
    if (threadIdx.x < M) {
      const int m = threadIdx.x;
      float bv = kNegInf;
      int bi = 0x7fffffff;
      for (int k = 0; k < ntc; ++k)
        if (better(s_am_v[k][m], s_am_i[k][m], bv, bi)) { bv = s_am_v[k][m]; bi = s_am_i[k][m]; }
      epi.am_val[static_cast<size_t>(m) * gridDim.x + blockIdx.x] = bv;
      epi.am_idx[static_cast<size_t>(m) * gridDim.x + blockIdx.x] = bi;
    }
  }
}

template <int BITS, int NT8, int EPI>
cudaError_t launch_t(const QTile& w, const ActIn& in, int M, const Epi& epi, const StepIO& io,
                     const SplitScratch& scr, bool pdl, cudaStream_t st) {
  auto kern = gemv_kernel<BITS, NT8, EPI>;
  const int ntc = kWarps / w.ksw;
  const size_t smem = gemv_smem_bytes(w, NT8, Pipe<BITS>::kItems);
  if (smem > kGemvMaxSmem) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((w.n_tiles + ntc - 1) / ntc, w.ksg, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, w, in, M, epi, io, scr.part);
}

template <int BITS, int NT8>
cudaError_t dispatch_epi(EpiKind kind, const QTile& w, const ActIn& in, int M, const Epi& epi,
                         const StepIO& io, const SplitScratch& scr, bool pdl, cudaStream_t st) {
  switch (kind) {
    case EPI_STORE: return launch_t<BITS, NT8, EPI_STORE>(w, in, M, epi, io, scr, pdl, st);
    case EPI_QKV: return launch_t<BITS, NT8, EPI_QKV>(w, in, M, epi, io, scr, pdl, st);
    case EPI_RESID: return launch_t<BITS, NT8, EPI_RESID>(w, in, M, epi, io, scr, pdl, st);
    case EPI_SWIGLU: return launch_t<BITS, NT8, EPI_SWIGLU>(w, in, M, epi, io, scr, pdl, st);
    case EPI_LOGITS: return launch_t<BITS, NT8, EPI_LOGITS>(w, in, M, epi, io, scr, pdl, st);
  }
  return cudaErrorInvalidValue;
}

template <int BITS>
cudaError_t dispatch_nt(EpiKind kind, const QTile& w, const ActIn& in, int M, const Epi& epi,
                        const StepIO& io, const SplitScratch& scr, bool pdl, cudaStream_t st) {
  if (M <= 8) return dispatch_epi<BITS, 1>(kind, w, in, M, epi, io, scr, pdl, st);
  return dispatch_epi<BITS, 2>(kind, w, in, M, epi, io, scr, pdl, st);
}

template <int BITS, int NT8>
cudaError_t set_attrs_nt() {
  const int v = static_cast<int>(kGemvMaxSmem);
  const auto a = cudaFuncAttributeMaxDynamicSharedMemorySize;
  cudaError_t e = cudaFuncSetAttribute(gemv_kernel<BITS, NT8, EPI_STORE>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<BITS, NT8, EPI_QKV>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<BITS, NT8, EPI_RESID>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<BITS, NT8, EPI_SWIGLU>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<BITS, NT8, EPI_LOGITS>, a, v);
  return e;
}

}  // namespace

cudaError_t gemv_init_attrs() {
  cudaError_t e = set_attrs_nt<4, 1>();
  if (e == cudaSuccess) e = set_attrs_nt<4, 2>();
  if (e == cudaSuccess) e = set_attrs_nt<8, 1>();
  if (e == cudaSuccess) e = set_attrs_nt<8, 2>();
  if (e == cudaSuccess) e = set_attrs_nt<16, 1>();
  if (e == cudaSuccess) e = set_attrs_nt<16, 2>();
  return e;
}

cudaError_t launch_gemv(const QTile& w, const ActIn& in_, int M, EpiKind kind, const Epi& epi_,
                        const StepIO& io, const SplitScratch& scr, bool pdl, cudaStream_t st) {
  if (M < 1 || M > kMaxRows) return cudaErrorInvalidValue;
  ActIn in = in_;
  set_vec(in);
  Epi epi = epi_;
  if (epi.res.x) set_vec(epi.res);
  if (w.ksg > 1) {
    const size_t need = static_cast<size_t>(w.ksg) * (w.n_tiles + kWarps) * kWarp * 8;
    if (scr.part == nullptr || scr.part_floats < need || w.counters == nullptr) return cudaErrorInvalidValue;
  }
  switch (w.bits) {
    case 4: return dispatch_nt<4>(kind, w, in, M, epi, io, scr, pdl, st);
    case 8: return dispatch_nt<8>(kind, w, in, M, epi, io, scr, pdl, st);
    case 16: return dispatch_nt<16>(kind, w, in, M, epi, io, scr, pdl, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace alm
