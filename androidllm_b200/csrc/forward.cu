// Persistent forward kernel: one launch runs a whole forward of up to eight
// activation rows (embedding, every layer, final norm, head, argmax).
//
// The grid holds as many CTAs as can be resident at once (two per SM), and
// every CTA walks the same list of phases:
//
//   embed | per layer: QKV+RoPE+KV write | scores | P.V | O+residual |
//           gate/up+SwiGLU | down+residual | final norm | head | argmax
//
// A phase is the grid of the corresponding standalone kernel, run as
// "virtual blocks" (vb = blockIdx.x, blockIdx.x + gridDim.x, ...) through the
// same device bodies, so the results are bit-identical to the standalone
// launches.  Phases are separated by a grid barrier instead of a kernel
// boundary, and a CTA issues the bulk copies of its next GEMV phase's first
// weight records before it waits at that barrier: the weight stream does not
// stop between phases, and no launch latency is paid between them.
//
// Grid barrier: a 64-bit arrival counter per model, never reset.  Each
// launch adds exactly kBarRound * gridDim.x to it (every CTA arrives once per
// barrier, then adds the rest of its kBarRound at exit), so a CTA finds the
// launch's base as the counter rounded down to that multiple.  Launches on
// the counter must not overlap (plain stream order).  Waits are bounded in
// time; a wait that gives up sets the error word to 3 and the CTA stops
// waiting for the rest of the launch.
#include <mutex>

#include "attn_body.cuh"
#include "forward.cuh"
#include "gemv_body.cuh"
#include "rows_body.cuh"

namespace alm {

__host__ __device__ int forward_barriers(int n_layers, bool head) { return 1 + 6 * n_layers + (head ? 2 : 0); }

namespace {

constexpr unsigned long long kBarWaitNs = 500ull * 1000 * 1000;

ALM_DEV unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
ALM_DEV unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Arrival: a release add, so every write the CTA made before (ordered by the
// preceding __syncthreads) is visible to whoever acquires the new count.
ALM_DEV void red_release_add(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
ALM_DEV void fence_acquire_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Shared state of the persistent kernel.
__shared__ unsigned long long s_bar_base;
__shared__ int s_broken;   // a barrier wait gave up: stop waiting

// Grid barrier on the per-model arrival counter.  Only `arrivals` lives in a
// register across phases; everything else comes from the parameters.
struct GridSync {
  const FwdParams& P;
  int arrivals = 0;
  int n_bar;

  ALM_DEV explicit GridSync(const FwdParams& p) : P(p), n_bar(forward_barriers(p.n_layers, p.do_head != 0)) {
    if (threadIdx.x == 0) {
      const unsigned long long span = static_cast<unsigned long long>(kBarRound) * gridDim.x;
      const unsigned long long v = ld_acquire_u64(P.bar);
      s_bar_base = v - v % span;
      s_broken = 0;
    }
    __syncthreads();
  }
  // All of the CTA's writes of the phase are done: publish them and arrive.
  ALM_DEV void arrive() {
    __syncthreads();
    ++arrivals;
    if (threadIdx.x == 0) {
      if (P.trace && arrivals <= n_bar)
        P.trace[static_cast<size_t>(arrivals - 1) * gridDim.x + blockIdx.x] = global_ns();
      red_release_add(P.bar, 1ull);
    }
  }
  // Wait until every CTA has arrived as often as this one.
  ALM_DEV void wait() {
    if (threadIdx.x == 0 && !s_broken) {
      // relaxed polls with a short sleep keep the pollers off the counter's
      // L2 slice; one acquire fence once the count is reached
      const unsigned long long target = s_bar_base + static_cast<unsigned long long>(arrivals) * gridDim.x;
      if (ld_relaxed_u64(P.bar) < target) {
        const unsigned long long t0 = global_ns();
        unsigned i = 0;
        while (ld_relaxed_u64(P.bar) < target) {
          __nanosleep(32);
          if ((++i & 63) == 0 && global_ns() - t0 > kBarWaitNs) {
            s_broken = 1;
            if (P.io.err) atomicExch(P.io.err, 3);
            break;
          }
        }
      }
      fence_acquire_gpu();
      if (P.trace && blockIdx.x == 0 && arrivals >= 1 && arrivals <= n_bar)
        P.trace[static_cast<size_t>(n_bar) * gridDim.x + arrivals - 1] = global_ns();
    }
    __syncthreads();
  }
  // Complete this launch's share of the counter.
  ALM_DEV void finish() {
    if (threadIdx.x == 0) atomicAdd(P.bar, static_cast<unsigned long long>(kBarRound - arrivals));
  }
};

union FwdShared {
  GemvShared<1> g;
  AttnShared a;
  RowShared r;
};
__shared__ FwdShared s_fwd;
__shared__ __align__(8) uint64_t s_bars[kGemvWarps * kSlots];

// The current phase's operands, written by thread 0 at the start of the
// phase: the body reads fields from here when it needs them instead of
// holding them in registers across its streamed main loop.
struct PhaseDesc {
  QTile w;
  ActIn in;
  Epi e;
  AttnArgs a;
};
__shared__ PhaseDesc s_desc;

// Dynamic shared memory: the weight-ring slots, then the GEMV activation
// staging.  Attention and row phases reuse it from offset 0 (no copy is in
// flight then).  The ring's mbarriers live in static shared memory, outside
// every reused region.
constexpr size_t kRingDataBytes = static_cast<size_t>(kGemvWarps) * kSlots * kMaxSlotBytes;
extern __shared__ __align__(128) unsigned char s_dyn[];

ALM_DEV Ring fwd_ring() {
  Ring r;
  r.base = s_dyn;
  r.bars = s_bars;
  r.slot_bytes = kMaxSlotBytes;
  return r;
}
ALM_DEV uint4* fwd_stage() { return reinterpret_cast<uint4*>(s_dyn + kRingDataBytes); }

ALM_DEV ActIn raw_act(const half* x, int ld, int H) {
  ActIn a;
  a.x = x;
  a.ld = ld;
  a.H = H;
  set_vec(a);
  return a;
}
ALM_DEV ActIn deferred_act(const FwdParams& P, const half* s, const float* ss, const half* w) {
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
// Input of layer li: the embedding rows, or the previous layer's residual
// sum with its post-attention-block norm deferred.
ALM_DEV ActIn layer_input(const FwdParams& P, int li) {
  return li == 0 ? raw_act(P.embed.out, P.hidden, P.hidden)
                 : deferred_act(P, P.s2, P.ss2, P.layers[li - 1].n_post);
}
ALM_DEV ActIn attn_norm_input(const FwdParams& P, int li) {
  return deferred_act(P, P.s1, P.ss1, P.layers[li].n_in);
}

// One GEMV phase: prefetch the first virtual block's weights, wait for the
// inputs, run the CTA's virtual blocks, arrive.
template <int BITS, int EPI>
ALM_DEV void gemv_phase_t(const FwdParams& P, GridSync& gs, uint32_t& seq, const QTile& w, const ActIn& in,
                          const Epi& epi) {
  constexpr int IPS = Pipe<BITS>::kItems;
  const Ring ring = fwd_ring();
  const int gx = gemv_grid_x(w);
  const int nvb = gx * w.ksg;
  int vb = blockIdx.x;
  GemvPlan plan;
  if (vb < nvb) {
    plan = gemv_plan(w, IPS, vb % gx, vb / gx, gx);
    gemv_issue_first<BITS>(ring, w, plan, seq);
  }
  gs.wait();
  while (vb < nvb) {
    seq += static_cast<uint32_t>(
        gemv_run<BITS, BITS == 16 ? 0 : 1, 1, EPI>(w, in, P.M, epi, P.io, P.part, plan, ring, seq, fwd_stage(),
                                                   s_fwd.g));
    vb += gridDim.x;
    if (vb < nvb) {
      __syncthreads();
      plan = gemv_plan(w, IPS, vb % gx, vb / gx, gx);
      gemv_issue_first<BITS>(ring, w, plan, seq);
    }
  }
  gs.arrive();
}

// Runs the GEMV phase described by s_desc (thread 0 has just written it).
template <int EPI>
ALM_DEV void gemv_phase(const FwdParams& P, GridSync& gs, uint32_t& seq) {
  __syncthreads();
  const int bits = s_desc.w.bits;
  if (bits == 4)
    gemv_phase_t<4, EPI>(P, gs, seq, s_desc.w, s_desc.in, s_desc.e);
  else if (bits == 8)
    gemv_phase_t<8, EPI>(P, gs, seq, s_desc.w, s_desc.in, s_desc.e);
  else
    gemv_phase_t<16, EPI>(P, gs, seq, s_desc.w, s_desc.in, s_desc.e);
}

ALM_DEV AttnArgs attn_args(const FwdParams& P, int li) {
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
  a.M = P.M;
  a.pos = P.io.pos;
  a.max_ctx = P.max_ctx;
  a.scores = P.scores;
  a.score_ld = P.score_ld;
  a.stats = P.stats;
  a.ctx = P.ctx;
  a.ldc = qdim;
  return a;
}

ALM_DEV void qkv_phase(const FwdParams& P, GridSync& gs, uint32_t& seq, int li) {
  if (threadIdx.x == 0) {
    Epi e;
    e.q = P.q;
    e.ldq = P.heads * P.head_dim;
    e.kcache = P.kcache + static_cast<size_t>(li) * P.kv_layer_elems;
    e.vcache = P.vcache + static_cast<size_t>(li) * P.kv_layer_elems;
    e.page_table = P.page_table;
    e.page_size = P.page_size;
    e.heads = P.heads;
    e.kv_heads = P.kv_heads;
    e.head_dim = P.head_dim;
    e.rope = P.rope;
    s_desc.e = e;
    s_desc.w = P.layers[li].qkv;
    s_desc.in = layer_input(P, li);
  }
  gemv_phase<EPI_QKV>(P, gs, seq);
}

ALM_DEV void attention_phases(const FwdParams& P, GridSync& gs, int li) {
  if (threadIdx.x == 0) s_desc.a = attn_args(P, li);
  gs.wait();   // also orders the descriptor write before every reader
  const AttnArgs& a = s_desc.a;
  const int ncm = attn_chunks_max(a);
  const int n_rg = attn_row_groups(a);
  const int kvh = a.kv_heads;
  const int n_chunks = (*a.pos + a.M + kAttnChunk - 1) / kAttnChunk;   // chunks holding positions
  const int nvb1 = n_chunks * kvh * n_rg;
  for (int vb = blockIdx.x; vb < nvb1; vb += gridDim.x) {
    attn_scores_pages(a, vb % n_chunks, s_dyn);
    __syncthreads();
    attn_scores_body(a, P.sqrt_hd, vb % n_chunks, (vb / n_chunks) % kvh, vb / (n_chunks * kvh), ncm, s_dyn,
                     s_fwd.a);
  }
  gs.arrive();
  gs.wait();
  const int nds = a.head_dim / 16, npg = attn_pv_groups(a);
  const int nvb2 = nds * kvh * npg;
  for (int vb = blockIdx.x; vb < nvb2; vb += gridDim.x) {
    attn_pv_pages(a, s_dyn);
    __syncthreads();
    attn_pv_body(a, ncm, vb % nds, (vb / nds) % kvh, vb / (nds * kvh), s_dyn, s_fwd.a);
  }
  gs.arrive();
}

// O projection + residual (sums of squares for the post-attention norm).
ALM_DEV void o_phase(const FwdParams& P, GridSync& gs, uint32_t& seq, int li) {
  if (threadIdx.x == 0) {
    Epi e;
    e.out = P.s1;
    e.ldo = P.hidden;
    e.n_out = P.hidden;
    e.res = layer_input(P, li);
    e.ss_out = P.ss1;
    s_desc.e = e;
    const int qdim = P.heads * P.head_dim;
    s_desc.w = P.layers[li].o;
    s_desc.in = raw_act(P.ctx, qdim, qdim);
  }
  gemv_phase<EPI_RESID>(P, gs, seq);
}

ALM_DEV void gu_phase(const FwdParams& P, GridSync& gs, uint32_t& seq, int li) {
  if (threadIdx.x == 0) {
    Epi e;
    e.out = P.h;
    e.ldo = P.inter;
    e.n_out = P.inter;
    s_desc.e = e;
    s_desc.w = P.layers[li].gu;
    s_desc.in = attn_norm_input(P, li);
  }
  gemv_phase<EPI_SWIGLU>(P, gs, seq);
}

ALM_DEV void down_phase(const FwdParams& P, GridSync& gs, uint32_t& seq, int li) {
  if (threadIdx.x == 0) {
    Epi e;
    e.out = P.s2;
    e.ldo = P.hidden;
    e.n_out = P.hidden;
    e.res = attn_norm_input(P, li);
    e.ss_out = P.ss2;
    s_desc.e = e;
    s_desc.w = P.layers[li].down;
    s_desc.in = raw_act(P.h, P.inter, P.inter);
  }
  gemv_phase<EPI_RESID>(P, gs, seq);
}

ALM_DEV void head_phase(const FwdParams& P, GridSync& gs, uint32_t& seq) {
  if (threadIdx.x == 0) {
    Epi e;
    e.out = P.logits;
    e.ldo = P.vocab;
    e.n_out = P.vocab;
    e.am_val = P.am_val;
    e.am_idx = P.am_idx;
    s_desc.e = e;
    s_desc.w = P.head;
    s_desc.in = raw_act(P.xn, P.hidden, P.hidden);
  }
  gemv_phase<EPI_LOGITS>(P, gs, seq);
}

__global__ void __launch_bounds__(kGemvThreads, 1) forward_kernel(const __grid_constant__ FwdParams P) {
  ring_init(fwd_ring());
  GridSync gs(P);
  uint32_t seq = 0;   // chunks through this warp's weight ring

  for (int vb = blockIdx.x; vb < P.M; vb += gridDim.x) embed_body(P.embed, vb);
  gs.arrive();

  for (int li = 0; li < P.n_layers; ++li) {
    qkv_phase(P, gs, seq, li);
    attention_phases(P, gs, li);
    o_phase(P, gs, seq, li);
    gu_phase(P, gs, seq, li);
    down_phase(P, gs, seq, li);
  }

  if (P.do_head) {
    gs.wait();
    const ActIn fin = layer_input(P, P.n_layers);
    for (int vb = blockIdx.x; vb < P.M; vb += gridDim.x)
      rownorm_body(fin, P.final_norm, P.eps, P.xn, P.hidden, vb, reinterpret_cast<half*>(s_dyn), s_fwd.r);
    gs.arrive();
    head_phase(P, gs, seq);
    gs.wait();
    for (int vb = blockIdx.x; vb < P.M; vb += gridDim.x)
      argmax_final_body(P.am_val, P.am_idx, gemv_grid_x(P.head), P.argmax, vb, s_fwd.r);
  }
  gs.finish();
}

}  // namespace

size_t forward_smem_bytes(size_t max_stage_bytes, int head_dim, int hidden) {
  size_t s = kRingDataBytes + max_stage_bytes;
  s = s > attn_pv_smem() ? s : attn_pv_smem();
  s = s > attn_scores_smem(head_dim) ? s : attn_scores_smem(head_dim);
  const size_t rn = static_cast<size_t>(hidden) * sizeof(half);
  return s > rn ? s : rn;
}

cudaError_t forward_init_attrs(size_t smem_bytes, int* ctas_per_sm) {
  // The limit is per device and only grows: models with smaller needs keep
  // the larger limit another model set.
  static std::mutex mu;
  static size_t set_bytes[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (smem_bytes > set_bytes[dev]) {
      e = cudaFuncSetAttribute(forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem_bytes));
      if (e != cudaSuccess) return e;
      set_bytes[dev] = smem_bytes;
    }
  }
  // The kernel calls non-inlined phase functions: make sure the per-thread
  // stack covers its frame (the driver also grows it at launch when needed).
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, forward_kernel);
  if (e != cudaSuccess) return e;
  size_t stack = 0;
  e = cudaDeviceGetLimit(&stack, cudaLimitStackSize);
  if (e != cudaSuccess) return e;
  const size_t need = (fa.localSizeBytes + 255) / 256 * 256;
  if (need > stack) {
    e = cudaDeviceSetLimit(cudaLimitStackSize, need);
    if (e != cudaSuccess) return e;
  }
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas_per_sm, forward_kernel, kGemvThreads, smem_bytes);
}

cudaError_t launch_forward(const FwdParams& p, int grid, size_t smem_bytes, cudaStream_t st) {
  forward_kernel<<<grid, kGemvThreads, smem_bytes, st>>>(p);
  return cudaGetLastError();
}

}  // namespace alm
