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
constexpr size_t kGemvMaxSmem = 200 * 1024;   // x staging limit (dynamic shared memory)

template <int BITS>
struct Pipe { static constexpr int U = BITS == 4 ? 8 : BITS == 8 ? 4 : 2; };

// Chunks of 8 activation columns staged per thread per batch (all loads of a
// batch are issued before any is used, so a batch costs one memory round trip).
constexpr int kStageBatch = 4;

ALM_DEV bool better(float v1, int i1, float v2, int i2) {
  return v1 > v2 || (v1 == v2 && i1 < i2);
}

template <int BITS, int NT8, int EPI>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(QTile w, ActIn in, int M, Epi epi, StepIO io,
                                                        float* __restrict__ part) {
  extern __shared__ uint4 xs[];  // [kb_local][NT8][2][32] uint4
  __shared__ float red[kWarps][kWarp][NT8 * 4];
  __shared__ float s_den_in[kMaxRows];
  __shared__ float s_den_res[kMaxRows];
  __shared__ int s_last;
  __shared__ float s_am_v[kWarps][NT8 * 8];
  __shared__ int s_am_i[kWarps][NT8 * 8];

  constexpr int V = QTileTraits<BITS>::kVec;
  constexpr int U = Pipe<BITS>::U;
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

  // ---- weight prefetch (does not depend on the previous kernel) ----------
  uint4 buf[U][V];
  uint32_t sbuf[U][2];
  auto load_kb = [&](int u, int kb) {
#pragma unroll
    for (int v = 0; v < V; ++v) buf[u][v] = ld_stream(qtile_ptr<BITS>(w.data, w.k_blocks, tile, kb, v, lane));
    if constexpr (BITS != 16) {
      const size_t sbase = static_cast<size_t>(tile) * w.nsb;
      sbuf[u][0] = ld_nc_u32(w.scales + (sbase + scale_block(w.block, kb, 0)) * 8 + g);
      sbuf[u][1] = w.block == 32 ? ld_nc_u32(w.scales + (sbase + scale_block(w.block, kb, 2)) * 8 + g)
                                 : sbuf[u][0];
    }
  };
#pragma unroll
  for (int u = 0; u < U; ++u)
    if (u < n) load_kb(u, kb0 + u);

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
  float acc[NT8][4];
#pragma unroll
  for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[nt][j] = 0.f;

  for (int base = 0; base < n; base += U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u;
      if (i < n) {
        uint4 cur[V];
#pragma unroll
        for (int v = 0; v < V; ++v) cur[v] = buf[u][v];
        const uint32_t sc0 = sbuf[u][0], sc1 = sbuf[u][1];
        if (i + U < n) load_kb(u, kb0 + i + U);
        const int kbl = kb0 + i - cta_kb0;
        uint4 xf[NT8][2];
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt) {
          const bool live = nt * 8 + g < M;   // B column g of n8 tile nt is activation row nt*8+g
          xf[nt][0] = live ? xs[((kbl * NT8 + nt) * 2 + 0) * kWarp + lane] : make_uint4(0, 0, 0, 0);
          xf[nt][1] = live ? xs[((kbl * NT8 + nt) * 2 + 1) * kWarp + lane] : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const half2 sc = u2h(s >= 2 ? sc1 : sc0);
          uint32_t a0, a1, a2, a3;
          decode_step<BITS>(cur, s, __low2half2(sc), __high2half2(sc), a0, a1, a2, a3);
#pragma unroll
          for (int nt = 0; nt < NT8; ++nt) {
            const uint4& X = xf[nt][s >> 1];
            const uint32_t b0 = (s & 1) ? X.z : X.x;
            const uint32_t b1 = (s & 1) ? X.w : X.y;
            mma16816(acc[nt], a0, a1, a2, a3, b0, b1);
          }
        }
      }
    }
  }

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
  const int cta_nkb = std::min(w.ksw * w.kps, w.k_blocks);
  const size_t smem = static_cast<size_t>(cta_nkb) * NT8 * 2 * kWarp * sizeof(uint4);
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
