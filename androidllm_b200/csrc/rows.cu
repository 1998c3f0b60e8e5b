// Row kernels of the forward: embedding gather, materialised RMSNorm(s) and
// the final argmax over per-CTA partials of the logits GEMV (bodies in
// rows_body.cuh).
#include "rows_body.cuh"

namespace alm {
namespace {

__global__ void __launch_bounds__(kRowThreads) embed_kernel(EmbedArgs a) {
  grid_dep_wait();
  embed_body(a, blockIdx.x);
}

__global__ void __launch_bounds__(kRowThreads) rownorm_kernel(ActIn in, const half* w2, float eps2, half* out,
                                                              int ldo) {
  extern __shared__ __align__(16) half xrow[];
  __shared__ RowShared sh;
  grid_dep_wait();
  rownorm_body(in, w2, eps2, out, ldo, blockIdx.x, xrow, sh);
}

__global__ void __launch_bounds__(kRowThreads) argmax_final_kernel(const float* am_val, const int* am_idx,
                                                                   int n_part, int* out) {
  __shared__ RowShared sh;
  grid_dep_wait();
  argmax_final_body(am_val, am_idx, n_part, out, blockIdx.x, sh);
}

// One row per block: out = fp16(res + fp16(o)) and the tile sums of squares
// in the RESID epilogue's order (per 16-column tile, lane g of 8 adds the
// squares of columns g and g + 8, then a butterfly over g).  o: the fp32
// sums of a row-split projection (tensor parallelism) or the fp16 outputs of
// the dense path (batched prefill), row stride H.
ALM_DEV float resid_operand(float v) { return round_h(v); }
ALM_DEV float resid_operand(half v) { return __half2float(v); }

// Row m: out = fp16(res + operand(col)) and the tile sums of squares in the
// RESID epilogue's order; operand(col) is the projection's value (fp32,
// rounded to fp16 like the epilogue's accumulator).
template <typename Operand>
ALM_DEV void resid_row(const ActIn& res, int m, int H, half* out, float* ss_out, Operand operand) {
  __shared__ float s_den;
  if (res.ss && threadIdx.x < kWarp) {
    const float d = row_denominator(res, m);
    if (threadIdx.x == 0) s_den = d;
  }
  body_sync();
  const int n_tiles = (H + 15) / 16;
  for (int base = 0; base < n_tiles * 8; base += kRowThreads) {
    const int e = base + static_cast<int>(threadIdx.x);
    const bool live = e < n_tiles * 8;
    const int tile = e / 8, g = e % 8;
    float sq = 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int col = tile * 16 + g + 8 * r;
      if (live && col < H) {
        const float rv = __half2float(__ldcg(res.x + static_cast<size_t>(m) * res.ld + col));
        const float rval = res.ss ? norm_value(rv, s_den, __half2float(__ldg(res.w + col))) : rv;
        const half s16 = __float2half_rn(fadd(rval, operand(col)));
        out[static_cast<size_t>(m) * H + col] = s16;
        const float sf = __half2float(s16);
        sq = r == 0 ? fmul(sf, sf) : fadd(sq, fmul(sf, sf));
      }
    }
    sq = fadd(sq, __shfl_xor_sync(0xffffffffu, sq, 1));
    sq = fadd(sq, __shfl_xor_sync(0xffffffffu, sq, 2));
    sq = fadd(sq, __shfl_xor_sync(0xffffffffu, sq, 4));
    if (live && g == 0) ss_out[static_cast<size_t>(m) * n_tiles + tile] = sq;
  }
}

// resid_rows_kernel<half> on row m, then the RMSNorm of its result (what
// rownorm_kernel computes from it, bit for bit: the same denominator from
// the same tile sums of squares, the same rounding), written to xout.
__global__ void __launch_bounds__(kRowThreads) resid_norm_kernel(ActIn res, const half* o16, int H, half* out,
                                                                 float* ss_out, ActIn nrm, half* xout, int ldx) {
  __shared__ float s_den2;
  grid_dep_wait();
  const int m = blockIdx.x;
  const half* row = o16 + static_cast<size_t>(m) * H;
  resid_row(res, m, H, out, ss_out, [&](int col) { return resid_operand(__ldcg(row + col)); });
  __syncthreads();   // the row and its tile sums are written (global, visible to the block)
  if (threadIdx.x < kWarp) {
    const float d = row_denominator(nrm, m);
    if (threadIdx.x == 0) s_den2 = d;
  }
  __syncthreads();
  const float den = s_den2;
  for (int k = threadIdx.x; k < H; k += kRowThreads) {
    const float v = __half2float(__ldcg(out + static_cast<size_t>(m) * H + k));
    xout[static_cast<size_t>(m) * ldx + k] = __float2half_rn(norm_value(v, den, __half2float(__ldg(nrm.w + k))));
  }
  grid_dep_launch();
}

template <typename OT>
__global__ void __launch_bounds__(kRowThreads) resid_rows_kernel(ActIn res, const OT* o32, int H, half* out,
                                                                 float* ss_out) {
  grid_dep_wait();
  const int m = blockIdx.x;
  const OT* row = o32 + static_cast<size_t>(m) * H;
  resid_row(res, m, H, out, ss_out, [&](int col) { return resid_operand(__ldcg(row + col)); });
  grid_dep_launch();
}

// Tensor parallelism over peer memory: block m sends row m of this rank's
// fp32 partial to every peer's receive slot (parity = the row's call count
// & 1, so a peer one call ahead writes the other slot), raises the peer's
// flag for (this rank, row m) to count + 1 with a system-scope release,
// waits (bounded) for every peer's flag, and adds the ranks' rows in rank
// order — the same sum on every rank — before the residual.
ALM_DEV void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
ALM_DEV unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kRowThreads) tp_p2p_resid_kernel(ActIn res, const float* o32, int H, half* out,
                                                                   float* ss_out, TpP2p p) {
  __shared__ unsigned s_epoch;
  grid_dep_wait();
  const int m = blockIdx.x;
  if (threadIdx.x == 0) s_epoch = p.counters[m];
  __syncthreads();
  const unsigned epoch = s_epoch, val = epoch + 1;
  const int parity = static_cast<int>(epoch & 1u);
  const float* mine = o32 + static_cast<size_t>(m) * H;
  // send row m to every peer: slot (parity, this rank, m) of its area
  for (int r = 0; r < p.world; ++r) {
    if (r == p.rank) continue;
    float* dst = tp_p2p_data(p, p.areas[r], parity, p.rank, m);
    for (int c = threadIdx.x; c < H; c += kRowThreads) dst[c] = __ldcg(mine + c);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < p.world; ++r)
      if (r != p.rank) st_release_sys(tp_p2p_flag(p, p.areas[r], parity, p.rank, m), val);
    // wait for every peer's row m in this rank's own area
    for (int r = 0; r < p.world; ++r) {
      if (r == p.rank) continue;
      const unsigned* f = tp_p2p_flag(p, p.areas[p.rank], parity, r, m);
      long long spins = 0;
      while (ld_acquire_sys(f) < val) {
        if (++spins > kTpP2pSpinLimit) {
          if (p.err) atomicExch(p.err, 2);
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncthreads();
  resid_row(res, m, H, out, ss_out, [&](int col) {
    float v = 0.f;
    for (int r = 0; r < p.world; ++r) {
      const float x = r == p.rank ? __ldcg(mine + col) : __ldcg(tp_p2p_data(p, p.areas[p.rank], parity, r, m) + col);
      v = r == 0 ? x : fadd(v, x);
    }
    return round_h(v);
  });
  __syncthreads();
  if (threadIdx.x == 0) p.counters[m] = val;
  grid_dep_launch();
}

__global__ void __launch_bounds__(kRowThreads) tp_argmax_local_kernel(const float* am_val, const int* am_idx,
                                                                      int n_part, int offset, int* pairs) {
  __shared__ RowShared sh;
  grid_dep_wait();
  const int m = blockIdx.x;
  float bv;
  int bi;
  argmax_reduce_body(am_val, am_idx, n_part, m, sh, bv, bi);
  if (threadIdx.x == 0) {
    pairs[2 * m] = __float_as_int(bv);
    pairs[2 * m + 1] = bi == 0x7fffffff ? 0x7fffffff : bi + offset;
  }
}

__global__ void __launch_bounds__(kWarp) tp_argmax_pick_kernel(const int* pairs, int world, int M, int* out) {
  grid_dep_wait();
  const int m = blockIdx.x;
  if (threadIdx.x != 0) return;
  float bv = kNegInf;
  int bi = 0x7fffffff;
  for (int r = 0; r < world; ++r) {
    const float v = __int_as_float(__ldcg(pairs + (static_cast<size_t>(r) * M + m) * 2));
    const int i = __ldcg(pairs + (static_cast<size_t>(r) * M + m) * 2 + 1);
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  out[m] = bi == 0x7fffffff ? 0 : bi;
}

__global__ void __launch_bounds__(kRowThreads) tp_logits_reorder_kernel(const half* gathered, int world, int M,
                                                                        int v_local, half* out) {
  grid_dep_wait();
  const int m = blockIdx.y, r = blockIdx.z;
  const half* src = gathered + (static_cast<size_t>(r) * M + m) * v_local;
  half* dst = out + static_cast<size_t>(m) * world * v_local + static_cast<size_t>(r) * v_local;
  for (int i = blockIdx.x * kRowThreads + threadIdx.x; i < v_local; i += gridDim.x * kRowThreads) dst[i] = src[i];
}

cudaLaunchConfig_t row_cfg(int M, size_t smem, bool pdl, cudaStream_t st, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(M);
  c.blockDim = dim3(kRowThreads);
  c.dynamicSmemBytes = smem;
  c.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return c;
}

}  // namespace

cudaError_t rows_init_attrs() {
  return cudaFuncSetAttribute(rownorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 24576 * 2);
}

cudaError_t launch_embed(const EmbedArgs& a, bool pdl, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = row_cfg(a.M, 0, pdl, st, attr);
  return cudaLaunchKernelEx(&c, embed_kernel, a);
}

cudaError_t launch_rownorm(const ActIn& in_, int M, const half* w2, float eps2, half* out, int ldo,
                           bool pdl, cudaStream_t st) {
  if (in_.H > 24576) return cudaErrorInvalidValue;
  ActIn in = in_;
  set_vec(in);
  cudaLaunchAttribute attr[1];
  const size_t smem = static_cast<size_t>(in.H) * sizeof(half);
  cudaLaunchConfig_t c = row_cfg(M, smem, pdl, st, attr);
  return cudaLaunchKernelEx(&c, rownorm_kernel, in, w2, eps2, out, ldo);
}

cudaError_t launch_argmax_final(const float* am_val, const int* am_idx, int n_part, int M, int* out,
                                bool pdl, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = row_cfg(M, 0, pdl, st, attr);
  return cudaLaunchKernelEx(&c, argmax_final_kernel, am_val, am_idx, n_part, out);
}

cudaError_t launch_tp_resid(const ActIn& res_, const float* o32, int M, int H, half* out, float* ss_out, bool pdl,
                            cudaStream_t st) {
  ActIn res = res_;
  set_vec(res);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = row_cfg(M, 0, pdl, st, attr);
  return cudaLaunchKernelEx(&c, resid_rows_kernel<float>, res, o32, H, out, ss_out);
}

cudaError_t launch_tp_p2p_resid(const ActIn& res_, const float* o32, int M, int H, half* out, float* ss_out,
                                const TpP2p& p, bool pdl, cudaStream_t st) {
  if (M < 1 || M > p.rows || H > p.row_floats || p.world < 2) return cudaErrorInvalidValue;
  ActIn res = res_;
  set_vec(res);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = row_cfg(M, 0, pdl, st, attr);
  return cudaLaunchKernelEx(&c, tp_p2p_resid_kernel, res, o32, H, out, ss_out, p);
}

cudaError_t launch_resid_norm(const ActIn& res_, const half* o16, int M, int H, half* out, float* ss_out,
                               const ActIn& nrm_, half* xout, int ldx, bool pdl, cudaStream_t st) {
  if (nrm_.ss != ss_out || nrm_.w == nullptr || nrm_.H != H) return cudaErrorInvalidValue;
  ActIn res = res_;
  set_vec(res);
  ActIn nrm = nrm_;
  set_vec(nrm);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = row_cfg(M, 0, pdl, st, attr);
  return cudaLaunchKernelEx(&c, resid_norm_kernel, res, o16, H, out, ss_out, nrm, xout, ldx);
}

cudaError_t launch_resid_rows16(const ActIn& res_, const half* o16, int M, int H, half* out, float* ss_out, bool pdl,
                                cudaStream_t st) {
  ActIn res = res_;
  set_vec(res);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = row_cfg(M, 0, pdl, st, attr);
  return cudaLaunchKernelEx(&c, resid_rows_kernel<half>, res, o16, H, out, ss_out);
}

cudaError_t launch_tp_argmax_local(const float* am_val, const int* am_idx, int n_part, int M, int offset,
                                   int* pairs, bool pdl, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = row_cfg(M, 0, pdl, st, attr);
  return cudaLaunchKernelEx(&c, tp_argmax_local_kernel, am_val, am_idx, n_part, offset, pairs);
}

cudaError_t launch_tp_argmax_pick(const int* pairs, int world, int M, int* out, bool pdl, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = row_cfg(M, 0, pdl, st, attr);
  c.blockDim = dim3(kWarp);
  return cudaLaunchKernelEx(&c, tp_argmax_pick_kernel, pairs, world, M, out);
}

cudaError_t launch_tp_logits_reorder(const half* gathered, int world, int M, int v_local, half* out, bool pdl,
                                     cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t c = row_cfg(M, 0, pdl, st, attr);
  c.gridDim = dim3((v_local + kRowThreads * 8 - 1) / (kRowThreads * 8), M, world);
  return cudaLaunchKernelEx(&c, tp_logits_reorder_kernel, gathered, world, M, v_local, out);
}

}  // namespace alm
