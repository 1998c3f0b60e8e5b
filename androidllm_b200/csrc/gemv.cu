// Standalone launches of the fused dequant-GEMV (one CTA per virtual block of
// the body in gemv_body.cuh) for forwards the persistent forward kernel does
// not run, alm_qmatmul and the shape benchmarks.
#include <algorithm>

#include "gemv_body.cuh"

namespace alm {
namespace {

constexpr size_t kGemvMaxSmem = 200 * 1024;   // dynamic shared memory limit per CTA

// Dynamic shared memory of one CTA: weight rings with their mbarriers, then
// the activation fragments.
inline size_t gemv_smem_bytes(const QTile& w, int rows) {
  return ring_bytes(gemv_slot_bytes(w)) + gemv_stage_bytes(w, rows);
}

// Split-K partials of one row group (floats).
__host__ __device__ inline size_t gemv_group_part_floats(const QTile& w) {
  return w.ksg <= 1 ? 0 : static_cast<size_t>(w.ksg) * (w.n_tiles + kGemvWarps) * kWarp * 8;
}

// M rows in row groups of kMaxRows: CTA x = (column block) * n_groups +
// group, so the CTAs that stream one weight tile for the different groups
// are neighbours in launch order and its later reads hit L2.  A group
// offsets every row-indexed pointer (activations and their norm partials,
// outputs, q, per-row positions, residual, sums of squares, argmax partials)
// and owns its split-K partials and column tickets.
template <int BITS, int SB, int NT8, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(QTile w, ActIn in, int M, Epi epi, StepIO io,
                                                            float* __restrict__ part) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ GemvShared<NT8> sh;
  const int slot_bytes = Pipe<BITS>::kItems * w.rec_u4 * 16;
  const Ring ring = ring_at(smem, slot_bytes);
  ring_init(ring);
  const int n_groups = (M + kMaxRows - 1) / kMaxRows;
  const int grp = blockIdx.x % n_groups, gx = gridDim.x / n_groups;
  const GemvPlan plan = gemv_plan(w, Pipe<BITS>::kItems, blockIdx.x / n_groups, blockIdx.y, gx);
  gemv_issue_first<BITS>(ring, w, plan, 0);
  uint4* xs = reinterpret_cast<uint4*>(smem + ring_bytes(slot_bytes));
  if (n_groups > 1) {
    const int r0 = grp * kMaxRows;
    M = min(kMaxRows, M - r0);
    in.x += static_cast<size_t>(r0) * in.ld;
    if (in.ss) in.ss += static_cast<size_t>(r0) * in.n_ss;
    if (epi.out) epi.out += static_cast<size_t>(r0) * epi.ldo;
    if (epi.out32) epi.out32 += static_cast<size_t>(r0) * epi.ldo;
    if (epi.q) epi.q += static_cast<size_t>(r0) * epi.ldq;
    if (epi.rows) epi.rows += r0;
    if (epi.res.x) epi.res.x += static_cast<size_t>(r0) * epi.res.ld;
    if (epi.res.ss) epi.res.ss += static_cast<size_t>(r0) * epi.res.n_ss;
    if (epi.ss_out) epi.ss_out += static_cast<size_t>(r0) * w.n_tiles;
    if (epi.am_val) epi.am_val += static_cast<size_t>(r0) * gx;
    if (epi.am_idx) epi.am_idx += static_cast<size_t>(r0) * gx;
    if (w.counters) w.counters += static_cast<size_t>(grp) * gx;
    if (part) part += static_cast<size_t>(grp) * gemv_group_part_floats(w);
  }
  // epilogue operands from earlier kernels, then the wait for the activations
  GemvPre<NT8> pre;
  gemv_prefetch<NT8, EPI>(w, M, epi, io, plan, sh, pre);
  grid_dep_wait();
  gemv_run<BITS, SB, NT8, EPI, true>(w, in, M, epi, io, part, plan, ring, 0, xs, sh, &pre);
}

template <int BITS, int NT8, int EPI>
cudaError_t launch_t(const QTile& w, const ActIn& in, int M, const Epi& epi, const StepIO& io,
                     const SplitScratch& scr, bool pdl, cudaStream_t st) {
  constexpr int SB1 = BITS == 16 ? 0 : 1;
  constexpr int SB2 = BITS == 16 ? 0 : 2;
  auto kern = w.sb == 2 ? gemv_kernel<BITS, SB2, NT8, EPI> : gemv_kernel<BITS, SB1, NT8, EPI>;
  const size_t smem = gemv_smem_bytes(w, M < kMaxRows ? M : kMaxRows);
  if (smem > kGemvMaxSmem) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gemv_grid_x(w) * ((M + kMaxRows - 1) / kMaxRows), w.ksg, 1);
  cfg.blockDim = dim3(kGemvThreads, 1, 1);
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
    case EPI_STORE32: return launch_t<BITS, NT8, EPI_STORE32>(w, in, M, epi, io, scr, pdl, st);
  }
  return cudaErrorInvalidValue;
}

template <int BITS>
cudaError_t dispatch_nt(EpiKind kind, const QTile& w, const ActIn& in, int M, const Epi& epi,
                        const StepIO& io, const SplitScratch& scr, bool pdl, cudaStream_t st) {
  if (M <= 8) return dispatch_epi<BITS, 1>(kind, w, in, M, epi, io, scr, pdl, st);
  return dispatch_epi<BITS, 2>(kind, w, in, M, epi, io, scr, pdl, st);
}

template <int BITS, int SB, int NT8>
cudaError_t set_attrs_sb() {
  const int v = static_cast<int>(kGemvMaxSmem);
  const auto a = cudaFuncAttributeMaxDynamicSharedMemorySize;
  cudaError_t e = cudaFuncSetAttribute(gemv_kernel<BITS, SB, NT8, EPI_STORE>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<BITS, SB, NT8, EPI_QKV>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<BITS, SB, NT8, EPI_RESID>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<BITS, SB, NT8, EPI_SWIGLU>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<BITS, SB, NT8, EPI_LOGITS>, a, v);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<BITS, SB, NT8, EPI_STORE32>, a, v);
  return e;
}

template <int BITS, int NT8>
cudaError_t set_attrs_nt() {
  if constexpr (BITS == 16) return set_attrs_sb<16, 0, NT8>();
  cudaError_t e = set_attrs_sb<BITS, 1, NT8>();
  if (e == cudaSuccess) e = set_attrs_sb<BITS, 2, NT8>();
  return e;
}

}  // namespace

cudaError_t gemv_init_attrs() {
  cudaError_t e = tc_gemv_init_attrs();
  if (e == cudaSuccess) e = set_attrs_nt<4, 1>();
  if (e == cudaSuccess) e = set_attrs_nt<4, 2>();
  if (e == cudaSuccess) e = set_attrs_nt<8, 1>();
  if (e == cudaSuccess) e = set_attrs_nt<8, 2>();
  if (e == cudaSuccess) e = set_attrs_nt<16, 1>();
  if (e == cudaSuccess) e = set_attrs_nt<16, 2>();
  return e;
}

size_t gemv_part_floats(const QTile& w, int rows) {
  if (w.layout == kLayoutRow) return tc_part_floats(w, rows);
  return gemv_group_part_floats(w) * static_cast<size_t>((rows + kMaxRows - 1) / kMaxRows);
}

int gemv_out_blocks(const QTile& w) { return w.layout == kLayoutRow ? w.n_rb : gemv_grid_x(w); }

cudaError_t launch_gemv(const QTile& w, const ActIn& in_, int M, EpiKind kind, const Epi& epi_,
                        const StepIO& io, const SplitScratch& scr, bool pdl, cudaStream_t st) {
  if (M < 1 || M > (w.layout == kLayoutRow ? kMaxDenseRows : kMaxPassRows)) return cudaErrorInvalidValue;
  // row groups past the first take their positions from epi.rows
  if (w.layout != kLayoutRow && M > kMaxRows && kind == EPI_QKV && epi_.rows == nullptr) return cudaErrorInvalidValue;
  ActIn in = in_;
  set_vec(in);
  Epi epi = epi_;
  if (epi.res.x) set_vec(epi.res);
  if (w.layout == kLayoutRow) return launch_tc_gemv(w, in, M, kind, epi, io, scr, pdl, st);
  if (w.ksg > 1) {
    if (scr.part == nullptr || scr.part_floats < gemv_part_floats(w, M) || w.counters == nullptr)
      return cudaErrorInvalidValue;
  }
  switch (w.bits) {
    case 4: return dispatch_nt<4>(kind, w, in, M, epi, io, scr, pdl, st);
    case 8: return dispatch_nt<8>(kind, w, in, M, epi, io, scr, pdl, st);
    case 16: return dispatch_nt<16>(kind, w, in, M, epi, io, scr, pdl, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace alm
