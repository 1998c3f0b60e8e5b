// C ABI of libandroidllm_b200: contexts, weights, models, paged KV cache,
// forward passes and the graph-replayed speculative step.
#include <cuda_profiler_api.h>

#include <algorithm>
#include <functional>
#include <map>
#include <tuple>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/androidllm_b200.h"
#include "common.cuh"
#include "cluster_fwd.cuh"
#include "forward.cuh"
#include "tp.cuh"
#include "gemv_body.cuh"
#include "kernels.cuh"

namespace alm {
cudaError_t launch_spec_prep_draft(const int* state, int* cand, const int* d_argmax, int i, int* tokens,
                                   int* pos, int prev_row, int refresh, cudaStream_t st);
cudaError_t launch_spec_prep_verify(const int* state, int* cand, const int* d_argmax, int k, int* tokens,
                                    int* pos, int prev_row, cudaStream_t st);
cudaError_t launch_spec_accept_greedy(int* state, const int* cand, const int* t_argmax, int k, int* out_tokens,
                                      int* out_accepted, int cap_tokens, int cap_steps, int sampled, cudaStream_t st);
}  // namespace alm

using namespace alm;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

#define ALM_CUDA(expr)                                                                         \
  do {                                                                                         \
    cudaError_t e_ = (expr);                                                                   \
    if (e_ != cudaSuccess) return fail(ALM_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)
#define ALM_REQ(cond, msg)                    \
  do {                                        \
    if (!(cond)) return fail(ALM_ERR_ARG, msg); \
  } while (0)
#define ALM_TRY(expr)        \
  do {                       \
    int rc_ = (expr);        \
    if (rc_ != ALM_OK) return rc_; \
  } while (0)

int n_sms_of(int device) {
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  return n;
}

int pow2_floor(int v) {
  int p = 1;
  while (p * 2 <= v) p *= 2;
  return p;
}

// Split-K launch shape of a weight.  Small matrices (a few hundred tiles or
// fewer) are latency-bound: spread them so the grid holds about two CTAs per
// SM, down to one k-block per warp, splitting K across CTAs when needed.
// Large matrices stream enough bytes per warp as they are: split K only
// inside the CTA and only as far as needed to reach two CTAs per SM.
void set_split(QTile& t, int ksw, int ksg) {
  t.ksw = ksw;
  const int s = ksw * ksg;
  t.kps = (t.k_blocks + s - 1) / s;
  // drop CTA rows that would get no k-blocks
  t.ksg = std::max(1, (((t.k_blocks + t.kps - 1) / t.kps) + ksw - 1) / ksw);
}

// Activation k-blocks one GEMV block may stage (64 KB of fragments at M <= 8).
constexpr int kMaxStageKb = 64;

// Launch shapes measured best on B200 (graph-replayed, PDL) for the step's
// shapes: narrow matrices let all 8 warps of a CTA split K and avoid cross-CTA
// splits (their ticket + reduction costs more than it saves) unless K is
// long; wide matrices give each warp whole tiles to stream.
void choose_split(QTile& t, int n_sms) {
  (void)n_sms;
  const int kb = t.k_blocks;
  int ksw, ksg;
  if (t.n_tiles > 2048) {
    ksw = 1;
    ksg = 1;
  } else if (t.n_tiles > 256) {
    ksw = 2;
    ksg = 1;
  } else if (kb > 100 && t.n_tiles >= 128) {
    ksw = 1;   // long K, enough tiles: one warp per tile, ~37 k-blocks per CTA
    ksg = (kb + 36) / 37;
  } else if (kb > 100) {
    ksw = 2;
    ksg = (kb + 11) / 12;
  } else {
    ksw = 8;
    ksg = (kb + 23) / 24;
  }
  ksw = std::min(ksw, std::max(1, pow2_floor(kb)));
  ksg = std::max(1, std::min(ksg, kb / ksw));
  set_split(t, ksw, ksg);
  while (t.ksw * t.kps > kMaxStageKb && t.ksw > 1) set_split(t, t.ksw / 2, t.ksg * 2);
}

// Row layout (tcgen05 GEMV): `wg` decoding warpgroups per CTA and `ksg` CTAs
// along K.  Up to 16 decoding warps fit an SM (tensor memory: 128 / 256 / 512
// columns for wg = 1 / 2 / 4), so wide matrices take one small CTA per 128
// rows and narrow ones split K until about one CTA per SM is busy.
void set_split_rows(QTile& t, int wg, int ksg) {
  t.wg = wg;
  t.ksw = 1;
  t.kps = (t.k_blocks + ksg - 1) / ksg;
  t.ksg = (t.k_blocks + t.kps - 1) / t.kps;
}

constexpr size_t kRowSmemBudget = 220 * 1024;

void choose_split_rows(QTile& t, int n_sms) {
  const int n_rb = t.n_rb, kb = t.k_blocks;
  int wg = 4, ksg = 1;
  if (n_rb >= 4 * n_sms) {
    wg = 1;
  } else if (n_rb >= 2 * n_sms) {
    wg = 2;
  } else if (n_rb < n_sms) {
    ksg = std::max(1, std::min((n_sms + n_rb / 2) / n_rb, kb / 4));
  }
  set_split_rows(t, wg, ksg);
  // activation staging for 16 rows beside the weight rings
  while (tc_gemv_smem_bytes(t, kMaxRows) > kRowSmemBudget && t.kps > 1) set_split_rows(t, wg, t.ksg + 1);
}

}  // namespace

// ----------------------------------------------------------------------------
// objects
// ----------------------------------------------------------------------------
struct alm_ctx {
  int device = 0;
  int n_sms = 148;
  cudaStream_t stream = nullptr;
  bool pdl = true;       // programmatic dependent launch between forward kernels
  bool persist = false;  // forwards of <= 8 rows as one persistent kernel
  bool cluster = false;  // single-row forwards of small models as one cluster kernel (opt-in)
  bool attn_decode = false;  // single-row attention as one kernel (opt-in: ALM_ATTN_DECODE=1)
  bool attn_fused = false;   // scores + P.V in one launch when the grid fits (opt-in: ALM_ATTN_FUSED=1)
  int tc = 0;            // row layout (tcgen05 GEMV): 0 never, 1 large weights, 2 always
  // models loaded from now on keep row-layout copies of their projections for
  // the batched prefill through the dense tcgen05 path (ALM_DENSE_PREFILL=0: off)
  bool dense_prefill = true;
  // tensor parallelism: NCCL communicator of this rank (alm_ctx_init_tp)
  void* tp_comm = nullptr;
  int tp_rank = 0, tp_world = 1;
  // peer-memory all-reduce of the row-split projections (alm_tp_p2p_*):
  // this rank's area, the peers' mapped areas, and whether it is in use
  TpP2p p2p;
  float* p2p_own = nullptr;
  bool p2p_ready = false, tp_p2p = false;
};

struct alm_qweight {
  alm_ctx* ctx = nullptr;
  QTile t;
  uint4* data = nullptr;
  unsigned* counters = nullptr;
  int out = 0, in = 0, in_real = 0;
};

namespace {

struct Layer {
  alm_qweight* qkv = nullptr;
  alm_qweight* o = nullptr;
  alm_qweight* gu = nullptr;
  alm_qweight* down = nullptr;
  half* n_in = nullptr;
  half* n_post = nullptr;
};

// Row-layout copies of a layer's projections for the dense prefill: q | k | v
// rows in order, gate rows then up rows (plain outputs, no fused epilogue).
struct DenseLayer {
  alm_qweight* qkv = nullptr;
  alm_qweight* o = nullptr;
  alm_qweight* gu = nullptr;
  alm_qweight* down = nullptr;
};

// Buffers of one prefill chunk of up to kMaxDenseRows rows.
struct PrefillWork {
  int rows = 0;                 // 0: not allocated
  int* tokens = nullptr;
  half* xa = nullptr;           // (rows, H) layer input, normalised
  half* xb = nullptr;           // (rows, H) attention block output, normalised
  half* qkv = nullptr;          // (rows, ld_qkv)
  float* q = nullptr;           // (rows, qd) after RoPE
  half* ctx = nullptr;          // (rows, qd) attention output
  half* o = nullptr;            // (rows, H) o / down outputs
  half* s = nullptr;            // (rows, H) residual sums
  float* ss = nullptr;          // (rows, H / 16) their sums of squares
  half* gu = nullptr;           // (rows, ld_gu) gate | up
  half* h = nullptr;            // (rows, ld_h)
  int ld_qkv = 0, ld_gu = 0, ld_h = 0;
  float* part = nullptr;        // split-K partials of the dense path
  size_t part_floats = 0;
  float* scores = nullptr;      // attention scratch for rows x max_ctx
  float* stats = nullptr;
  int attn_ctx = 0, score_ld = 0;
};

struct Work {
  int* tokens = nullptr;
  int* pos = nullptr;
  int* err = nullptr;
  half* x0 = nullptr;
  half* s1 = nullptr;
  half* s2 = nullptr;
  float* ss1 = nullptr;
  float* ss2 = nullptr;
  float* q = nullptr;
  half* ctx = nullptr;
  half* h = nullptr;
  half* xn = nullptr;
  half* xout = nullptr;
  half* logits = nullptr;
  float* am_val = nullptr;
  int* am_idx = nullptr;
  int n_am = 0;
  int* argmax = nullptr;
  float* part = nullptr;
  size_t part_floats = 0;
  float* sample_scratch = nullptr;   // kMaxRows * vocab fp32 for the sampler
  float* scores = nullptr;
  float* stats = nullptr;
  float* pv_part = nullptr;      // P.V span partials (contexts of several spans)
  unsigned* pv_ticket = nullptr;
  unsigned* fz_count = nullptr;  // one-launch attention: counts, tickets, chunk partials
  unsigned* fz_ticket = nullptr;
  float* fz_part = nullptr;
  // tensor parallelism
  float* o32 = nullptr;        // (kMaxRows, hidden) fp32 partials of the row-split projections
  int* tp_pairs = nullptr;     // (kMaxRows, 2) local argmax, then (world, kMaxRows, 2) gathered
  half* logits_local = nullptr;  // (kMaxRows, vocab_local) this rank's vocabulary slice
  half* logits_gather = nullptr; // (world, kMaxRows, vocab_local)
  int attn_ctx = 0;       // capacity of the attention scratch (positions)
  int score_ld = 0;       // row stride of the score scratch
  int* pinned = nullptr;  // host staging for small copies
  // multi-sequence passes: per row {position, page-table offset}, per sequence AttnSeq
  int2* rows = nullptr;
  AttnSeq* seqs = nullptr;
  double* u_rows = nullptr;      // (kMaxRows) uniforms of alm_model_sample_rows
  unsigned char* seq_host = nullptr;   // pinned staging of rows, sequences and tokens
};

int dev_alloc(void** p, size_t bytes) {
  if (bytes == 0) bytes = 16;
  ALM_CUDA(cudaMalloc(p, bytes));
  return ALM_OK;
}
template <typename T>
int dev_alloc_t(T** p, size_t count) {
  return dev_alloc(reinterpret_cast<void**>(p), count * sizeof(T));
}
void dev_free(void* p) {
  if (p) cudaFree(p);
}

// Device copies of a standalone call's inputs and outputs (freed on return).
struct DevBufs {
  std::vector<void*> ptrs;
  ~DevBufs() {
    for (void* p : ptrs) cudaFree(p);
  }
  template <typename T>
  int get(T** p, size_t count) {
    ALM_TRY(dev_alloc_t(p, count));
    ptrs.push_back(*p);
    return ALM_OK;
  }
};

}  // namespace

struct alm_model {
  alm_ctx* ctx = nullptr;
  alm_model_config cfg{};
  half* rope = nullptr;
  std::vector<Layer> layers;
  void* embed_table = nullptr;
  half* embed_scale = nullptr;
  int embed_bits = 0, embed_block = 0, embed_nsb = 0, embed_row_bytes = 0;
  alm_qweight* head = nullptr;   // owned
  half* final_norm = nullptr;
  bool finalized = false;
  Work ws;
  // persistent forward kernel
  FwdLayer* fwd_layers = nullptr;           // device, one per layer
  unsigned long long* fwd_bar = nullptr;    // device grid-barrier counter
  size_t fwd_smem = 0;
  int fwd_grid = 0;                         // 0: not available for this model
  // cluster forward kernel (single-row forwards)
  size_t cf_smem = 0;
  bool cf_ok = false;
  // tensor parallelism: this model is the rank's shard (local heads, FFN
  // slice, head rows [vocab_offset, vocab_offset + vocab_local))
  bool tp = false;
  int vocab_offset = 0, vocab_local = 0;
  bool tp_need_logits = false;   // gather the full logits after the head
  std::vector<DenseLayer> dense;   // per layer; qkv null: no dense copies
  // the forward being enqueued is a multi-sequence pass (ws.rows / ws.seqs)
  int ms_n_seq = 0, ms_n_rg = 0, ms_n_pg = 0;
  // captured multi-sequence passes: (the KV cache's buffers and geometry,
  // rows, sequences, row groups, P.V groups, head) -> graph.  Their inputs
  // are device arrays, so a pass of the same shape on the same buffers
  // replays the graph (cleared when the model's scratch is reallocated).
  using MsKey = std::tuple<const void*, const void*, const void*, int, int, int, int, int, int, int>;
  std::map<MsKey, cudaGraphExec_t> ms_graphs;
  PrefillWork pf;
  // attention passes enqueued now are known to fit one P.V span: launch the
  // unsplit P.V kernel even when the KV capacity is longer (speed only: the
  // unsplit kernel walks any context length)
  bool pv_one_span = false;
};

struct alm_kv {
  alm_ctx* ctx = nullptr;
  // n_slots sequences of max_len positions each; slot s's page numbers are
  // row s of the page table (pages_per_slot entries)
  int n_layers = 0, kv_heads = 0, head_dim = 0, page_size = 16, n_pages = 0, max_len = 0;
  int n_slots = 1, pages_per_slot = 0;
  size_t layer_elems = 0;
  half* k = nullptr;
  half* v = nullptr;
  int* page_table = nullptr;
};

struct alm_spec {
  alm_model* target = nullptr;
  alm_model* draft = nullptr;
  alm_kv* tkv = nullptr;
  alm_kv* dkv = nullptr;
  int k = 0;
  int* state = nullptr;      // device [4]
  int* cand = nullptr;       // device [k]
  int* out_tokens = nullptr; // device ring
  int* out_acc = nullptr;
  int cap_steps = 0, cap_tokens = 0;
  cudaGraphExec_t graph = nullptr;
  // the same step with the unsplit P.V kernel, replayed while every pass
  // fits one P.V span (null when neither KV cache is longer than a span)
  cudaGraphExec_t graph_short = nullptr;
  int* pinned = nullptr;     // host: 4 + cap_tokens + cap_steps
  int n_kernels = 0;         // kernel nodes in the step graph
  // sampling at temperature > 0 (engine.py:26-45 per draft and target row)
  float temperature = 0.f;   // <= 0: greedy
  float top_p = 1.f, min_p = 0.f;
  double* uniforms = nullptr;  // device stream of uniform draws; state[4] = next unused
  int n_uniforms = 0, cap_uniforms = 0;
  // min(1, p/q) rejection sampling instead of the reference's rule (T > 0)
  bool rejection = false;
  // the first draft forward re-forwards the token at pos - 1 (state[5])
  bool refresh = false;
  float* probs = nullptr;      // (k + 1) target rows then k draft rows of vocab fp32
};

namespace {

struct DeviceGuard {
  explicit DeviceGuard(int d) { cudaSetDevice(d); }
};

// --------------------------------------------------------------------------
// weight building
// --------------------------------------------------------------------------
size_t src_bytes(int bits, int rows, int k_pad) {
  return bits == 4 ? static_cast<size_t>(rows) * k_pad / 2
                   : bits == 8 ? static_cast<size_t>(rows) * k_pad : static_cast<size_t>(rows) * k_pad * 2;
}

// With mode 1, weights at least this large take the row layout (tcgen05
// kernel); smaller ones keep the mma.sync tile layout.
constexpr size_t kRowMinBytes = 4u << 20;
// pinned staging of a multi-sequence pass: rows, sequences, tokens
constexpr size_t kSeqStaging = kMaxPassRows * (sizeof(int2) + sizeof(AttnSeq) + sizeof(int));

bool use_rows(const alm_ctx* ctx, int bits, int block, int n_rows, int in) {
  if ((bits != 4 && bits != 8) || block % 64 != 0 || ctx->tc == 0) return false;
  return ctx->tc == 2 || static_cast<size_t>(n_rows) * in * bits / 8 >= kRowMinBytes;
}

int check_format(int bits, int block, int in, int in_real) {
  ALM_REQ(bits == 4 || bits == 8 || bits == 16, "bits must be 4, 8 or 16");
  ALM_REQ(in > 0 && in_real > 0 && in_real <= in, "invalid in / in_real");
  if (bits != 16) {
    ALM_REQ(block == 32 || (block > 0 && block % 64 == 0), "block must be 32 or a multiple of 64");
    ALM_REQ(in % block == 0, "in must be a multiple of block");
  }
  if (bits == 4) ALM_REQ(in % 2 == 0, "int4 rows need an even length");
  return ALM_OK;
}

// Build one weight from up to 3 sources with a destination row map for the
// chosen layout (dst row -> (src << 24) | src row, or -1).  `allow_rows`:
// the consumer's epilogue exists in the row layout (every one but QKV).
void free_dense(DenseLayer& D) {
  alm_qweight_free(D.qkv);
  alm_qweight_free(D.o);
  alm_qweight_free(D.gu);
  alm_qweight_free(D.down);
  D = DenseLayer{};
}

void free_prefill_work(PrefillWork& pf) {
  for (void* p : {(void*)pf.tokens, (void*)pf.xa, (void*)pf.xb, (void*)pf.qkv, (void*)pf.q, (void*)pf.ctx,
                  (void*)pf.o, (void*)pf.s, (void*)pf.ss, (void*)pf.gu, (void*)pf.h, (void*)pf.part,
                  (void*)pf.scores, (void*)pf.stats})
    dev_free(p);
  pf = PrefillWork{};
}

// Whether a layer's projections get row-layout copies for the dense prefill:
// int4 / int8 with 64-column blocks (the row layout's format), whole models
// only (a tensor-parallel shard prefills through its row-split forward).
bool dense_prefill_ok(const alm_model* m, const alm_proj_src* p) {
  if (!m->ctx->dense_prefill || m->tp) return false;
  for (int i = 0; i < 7; ++i)
    if ((p[i].bits != 4 && p[i].bits != 8) || p[i].block % 64 != 0) return false;
  return true;
}

// Every layer has its row-layout copies.
bool dense_ready(const alm_model* m) {
  for (const DenseLayer& D : m->dense)
    if (!D.qkv) return false;
  return !m->dense.empty();
}

int build_qweight(alm_ctx* ctx, const alm_proj_src* srcs, int n_src,
                  const std::function<std::vector<int>(int)>& map_of, int n_rows, bool allow_rows,
                  alm_qweight** out, bool force_rows = false) {
  const int bits = srcs[0].bits, block = srcs[0].block, in = srcs[0].in, in_real = srcs[0].in_real;
  for (int i = 0; i < n_src; ++i) {
    ALM_TRY(check_format(srcs[i].bits, srcs[i].block, srcs[i].in, srcs[i].in_real));
    ALM_REQ(srcs[i].bits == bits && srcs[i].in == in && srcs[i].in_real == in_real &&
                (bits == 16 || srcs[i].block == block),
            "fused projections must share bits, block and input size");
    ALM_REQ(srcs[i].packed_host != nullptr && (bits == 16 || srcs[i].scale_host != nullptr),
            "missing weight data");
  }
  auto* w = new alm_qweight();
  w->ctx = ctx;
  w->out = n_rows;
  w->in = in;
  w->in_real = in_real;
  QTile& t = w->t;
  t.bits = bits;
  t.block = bits == 16 ? 64 : block;
  t.n_rows = n_rows;
  t.n_tiles = (n_rows + 15) / 16;
  t.k_blocks = (in + 63) / 64;
  t.sb = bits == 16 ? 0 : (block == 32 ? 2 : 1);
  t.k_real = in_real;
  if (force_rows)
    ALM_REQ((bits == 4 || bits == 8) && block % 64 == 0, "the row layout takes int4 / int8 with 64-column blocks");
  const bool rows = force_rows || (allow_rows && use_rows(ctx, bits, block, n_rows, in));
  size_t n_rec = 0;
  int n_counters = 0;
  if (rows) {
    t.layout = kLayoutRow;
    t.n_rb = (n_rows + kRowBlock - 1) / kRowBlock;
    t.rec_u4 = ((bits == 4 ? 2 : 4) * 512 + 64) / 16;   // codes + 32 fp16 scales
    choose_split_rows(t, ctx->n_sms);
    n_rec = static_cast<size_t>(t.n_rb) * 4 * t.k_blocks;
    n_counters = t.n_rb;
  } else {
    choose_split(t, ctx->n_sms);
    const int vec = bits == 4 ? 1 : bits == 8 ? 2 : 4;
    t.rec_u4 = vec * kWarp + t.sb * 2;   // codes + 8 half2 scales (32 B) per set
    n_rec = static_cast<size_t>(t.n_tiles) * t.k_blocks;
    n_counters = (t.n_tiles + 8 / t.ksw - 1) / (8 / t.ksw) * kMaxRowGroups;   // per row group
  }
  const std::vector<int> dst_map = map_of(t.layout);
  // every destination row must name an existing source row: the repack
  // kernels index the sources with these entries unchecked
  ALM_REQ(dst_map.size() >= static_cast<size_t>(rows ? t.n_rb * kRowBlock : t.n_tiles * 16),
          "row map shorter than the layout");
  for (const int d : dst_map) {
    if (d < 0) continue;
    const int si = d >> 24, r = d & 0xffffff;
    ALM_REQ(si < n_src && r < srcs[si].out, "row map names a source row that does not exist");
  }
  std::vector<void*> tmp;
  auto cleanup = [&]() {
    for (void* p : tmp) cudaFree(p);
  };
  int rc = ALM_OK;
  const void* dsrc[3] = {nullptr, nullptr, nullptr};
  const half* dscale[3] = {nullptr, nullptr, nullptr};
  int* dmap = nullptr;
  do {
    if ((rc = dev_alloc_t(&w->data, n_rec * t.rec_u4)) != ALM_OK) break;
    for (int i = 0; i < n_src && rc == ALM_OK; ++i) {
      void* p = nullptr;
      const size_t nb = src_bytes(bits, srcs[i].out, in);
      if ((rc = dev_alloc(&p, nb)) != ALM_OK) break;
      tmp.push_back(p);
      if (cudaMemcpy(p, srcs[i].packed_host, nb, cudaMemcpyHostToDevice) != cudaSuccess) {
        rc = fail(ALM_ERR_CUDA, "weight upload failed");
        break;
      }
      dsrc[i] = p;
      if (bits != 16) {
        void* s = nullptr;
        const size_t sb = static_cast<size_t>(srcs[i].out) * (in / block) * sizeof(half);
        if ((rc = dev_alloc(&s, sb)) != ALM_OK) break;
        tmp.push_back(s);
        if (cudaMemcpy(s, srcs[i].scale_host, sb, cudaMemcpyHostToDevice) != cudaSuccess) {
          rc = fail(ALM_ERR_CUDA, "scale upload failed");
          break;
        }
        dscale[i] = static_cast<const half*>(s);
      }
    }
    if (rc != ALM_OK) break;
    if ((rc = dev_alloc_t(&dmap, dst_map.size())) != ALM_OK) break;
    tmp.push_back(dmap);
    if (cudaMemcpy(dmap, dst_map.data(), dst_map.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) {
      rc = fail(ALM_ERR_CUDA, "row map upload failed");
      break;
    }
    cudaError_t e = rows ? launch_repack_rows(dsrc, dscale, n_src, dmap, t, w->data, in, ctx->stream)
                         : launch_repack(dsrc, dscale, n_src, dmap, t, w->data, in, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
      rc = fail(ALM_ERR_CUDA, std::string("repack: ") + cudaGetErrorString(e));
      break;
    }
    if ((rc = dev_alloc_t(&w->counters, n_counters)) != ALM_OK) break;
    if (cudaMemset(w->counters, 0, n_counters * sizeof(unsigned)) != cudaSuccess) {
      rc = fail(ALM_ERR_CUDA, "counter init failed");
      break;
    }
  } while (false);
  cleanup();
  if (rc != ALM_OK) {
    alm_qweight_free(w);
    return rc;
  }
  t.data = w->data;
  t.counters = w->counters;
  *out = w;
  return ALM_OK;
}

// Destination rows of a layout: tiles of 16 or blocks of 128.
int padded_rows(int rows, int layout) {
  const int r = layout == kLayoutRow ? kRowBlock : 16;
  return (rows + r - 1) / r * r;
}

std::function<std::vector<int>(int)> identity_map(int rows) {
  return [rows](int layout) {
    std::vector<int> m(padded_rows(rows, layout), -1);
    for (int r = 0; r < rows; ++r) m[r] = r;
    return m;
  };
}

// Split-K scratch large enough for weight w (floats).
size_t split_need(const alm_qweight* w) { return w ? gemv_part_floats(w->t, kMaxPassRows) : 0; }

int ensure_part(Work& ws, size_t need) {
  if (need <= ws.part_floats) return ALM_OK;
  dev_free(ws.part);
  ws.part = nullptr;
  ws.part_floats = 0;
  ALM_TRY(dev_alloc_t(&ws.part, need));
  ws.part_floats = need;
  return ALM_OK;
}

int ensure_attn(alm_model* m, int max_ctx) {
  Work& ws = m->ws;
  if (max_ctx <= ws.attn_ctx && (!m->ctx->attn_fused || ws.fz_part)) return ALM_OK;
  max_ctx = std::max(max_ctx, ws.attn_ctx);
  for (auto& kvg : m->ms_graphs) cudaGraphExecDestroy(kvg.second);   // they hold the old scratch
  m->ms_graphs.clear();
  const int gq = m->cfg.heads / m->cfg.kv_heads;
  // row groups of the largest pass; a multi-sequence pass (up to kMaxPassRows
  // rows of up to kMaxRows sequences) starts a group per sequence, which
  // adds at most one per sequence
  const int n_rg = (kMaxPassRows * gq + kAttnRows - 1) / kAttnRows + kMaxRows;
  const int cap = (max_ctx + kAttnChunk - 1) / kAttnChunk * kAttnChunk;
  dev_free(ws.scores);
  dev_free(ws.stats);
  dev_free(ws.pv_part);
  dev_free(ws.pv_ticket);
  dev_free(ws.fz_count);
  dev_free(ws.fz_ticket);
  dev_free(ws.fz_part);
  ws.scores = nullptr;
  ws.stats = nullptr;
  ws.pv_part = nullptr;
  ws.pv_ticket = nullptr;
  ws.fz_count = nullptr;
  ws.fz_ticket = nullptr;
  ws.fz_part = nullptr;
  ws.attn_ctx = 0;
  // rows padded by one chunk: the P.V kernel reads whole 16-position groups
  const int ld = cap + kAttnChunk;
  ALM_TRY(dev_alloc_t(&ws.scores, static_cast<size_t>(m->cfg.kv_heads) * n_rg * kAttnRows * ld));
  ALM_TRY(dev_alloc_t(&ws.stats, static_cast<size_t>(m->cfg.kv_heads) * n_rg * (cap / kAttnChunk) * kAttnRows * 2));
  // P.V span split: (kv head, slice, group) keys x spans x kPvRows x 16 partials
  const size_t keys = static_cast<size_t>(m->cfg.kv_heads) * (m->cfg.head_dim / 16) *
                      ((kMaxRows * gq + kPvRows - 1) / kPvRows);
  ALM_TRY(dev_alloc_t(&ws.pv_part, keys * attn_pv_spans(cap) * kPvRows * 16));
  ALM_TRY(dev_alloc_t(&ws.pv_ticket, keys));
  ALM_CUDA(cudaMemset(ws.pv_ticket, 0, keys * sizeof(unsigned)));
  // one-launch attention (only on a context that enables it; without them
  // the layer takes the two passes): (kv head, row group) counters and
  // tickets, and a (kv head, row group, chunk) partial of 16 rows x head_dim
  if (m->ctx->attn_fused) {
    const size_t fz_keys = static_cast<size_t>(m->cfg.kv_heads) * n_rg;
    ALM_TRY(dev_alloc_t(&ws.fz_count, fz_keys));
    ALM_TRY(dev_alloc_t(&ws.fz_ticket, fz_keys));
    ALM_CUDA(cudaMemset(ws.fz_count, 0, fz_keys * sizeof(unsigned)));
    ALM_CUDA(cudaMemset(ws.fz_ticket, 0, fz_keys * sizeof(unsigned)));
    ALM_TRY(dev_alloc_t(&ws.fz_part, fz_keys * (cap / kAttnChunk) * kAttnRows * m->cfg.head_dim));
  }
  ws.attn_ctx = cap;
  ws.score_ld = ld;
  return ALM_OK;
}

// --------------------------------------------------------------------------
// forward enqueue (no host synchronisation)
// --------------------------------------------------------------------------
// ---- per-launch profile of a captured step (alm_spec_profile) ----------------
struct LaunchProfile {
  cudaStream_t st = nullptr;
  int role = 0;
  std::vector<cudaEvent_t> ev;
  std::vector<int> op, rows;
  cudaError_t err = cudaSuccess;
};
thread_local LaunchProfile* g_prof = nullptr;

void prof_role(int role) {
  if (g_prof) g_prof->role = role;
}

}  // namespace

namespace alm {
void prof_mark(int op, int rows) {
  LaunchProfile* p = g_prof;
  if (!p || p->err != cudaSuccess) return;
  cudaEvent_t e = nullptr;
  p->err = cudaEventCreate(&e);
  if (p->err != cudaSuccess) return;
  p->ev.push_back(e);
  p->op.push_back(op + 100 * p->role);
  p->rows.push_back(rows);
  p->err = cudaEventRecordWithFlags(e, p->st, cudaEventRecordExternal);
}
}  // namespace alm

namespace {

SplitScratch scratch_of(alm_model* m) { return SplitScratch{m->ws.part, m->ws.part_floats}; }

int n_h_tiles(const alm_model* m) { return (m->cfg.hidden + 15) / 16; }

ActIn raw_in(const half* x, int ld, int H) {
  ActIn a;
  a.x = x;
  a.ld = ld;
  a.H = H;
  return a;
}
ActIn deferred_in(const alm_model* m, const half* s, const float* ss, const half* w) {
  ActIn a;
  a.x = s;
  a.ld = m->cfg.hidden;
  a.ss = ss;
  a.n_ss = n_h_tiles(m);
  a.w = w;
  a.eps = m->cfg.rms_eps;
  a.H = m->cfg.hidden;
  return a;
}

#define ALM_LAUNCH(expr)                                                                             \
  do {                                                                                               \
    cudaError_t e_ = (expr);                                                                         \
    if (e_ != cudaSuccess) return fail(ALM_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)

// A row-split projection of a tensor-parallel shard: this rank's fp32
// partial sums over its K slice, an all-reduce (sum) over the ranks, then
// out = fp16(res + fp16(sum)) with the sums of squares of the next norm.
int enqueue_tp_rowsplit(alm_model* m, const alm_qweight* w, const ActIn& in, int M, const ActIn& res, half* out,
                        float* ss_out, bool pdl) {
  Work& ws = m->ws;
  cudaStream_t st = m->ctx->stream;
  const int H = m->cfg.hidden;
  Epi e;
  e.out32 = ws.o32;
  e.ldo = H;
  e.n_out = H;
  ALM_LAUNCH(launch_gemv(w->t, in, M, EPI_STORE32, e, StepIO{ws.pos, ws.err}, scratch_of(m), pdl, st));
  if (m->ctx->tp_p2p) {
    // one kernel: exchange over peer memory, rank-order sum, residual
    TpP2p p = m->ctx->p2p;
    p.err = ws.err;
    ALM_LAUNCH(launch_tp_p2p_resid(res, ws.o32, M, H, out, ss_out, p, pdl, st));
    return ALM_OK;
  }
  std::string err;
  if (tp_allreduce_sum_f32(m->ctx->tp_comm, ws.o32, static_cast<size_t>(M) * H, st, &err))
    return fail(ALM_ERR_CUDA, err);
  ALM_LAUNCH(launch_tp_resid(res, ws.o32, M, H, out, ss_out, false, st));
  return ALM_OK;
}

int enqueue_layer(alm_model* m, int li, alm_kv* kv, int M, const ActIn& in, bool pdl) {
  const alm_model_config& c = m->cfg;
  Layer& L = m->layers[li];
  Work& ws = m->ws;
  cudaStream_t st = m->ctx->stream;
  StepIO io{ws.pos, ws.err};
  const SplitScratch scr = scratch_of(m);
  const int qdim = c.heads * c.head_dim;

  Epi e;
  e.q = ws.q;
  e.ldq = qdim;
  e.kcache = kv->k + static_cast<size_t>(li) * kv->layer_elems;
  e.vcache = kv->v + static_cast<size_t>(li) * kv->layer_elems;
  e.page_table = kv->page_table;
  e.page_size = kv->page_size;
  e.heads = c.heads;
  e.kv_heads = c.kv_heads;
  e.head_dim = c.head_dim;
  e.rope = m->rope;
  if (m->ms_n_seq) e.rows = ws.rows;
  ALM_LAUNCH(launch_gemv(L.qkv->t, in, M, EPI_QKV, e, io, scr, pdl, st));
  prof_mark(ALM_OP_QKV, M);

  AttnArgs a;
  a.q = ws.q;
  a.ldq = qdim;
  a.kcache = e.kcache;
  a.vcache = e.vcache;
  a.page_table = kv->page_table;
  a.page_size = kv->page_size;
  a.heads = c.heads;
  a.kv_heads = c.kv_heads;
  a.head_dim = c.head_dim;
  a.M = M;
  a.pos = ws.pos;
  a.max_ctx = kv->max_len;
  a.scores = ws.scores;
  a.score_ld = ws.score_ld;
  a.stats = ws.stats;
  a.ctx = ws.ctx;
  a.ldc = qdim;
  a.pv_part = m->pv_one_span ? nullptr : ws.pv_part;
  a.pv_ticket = ws.pv_ticket;
  if (m->ms_n_seq) {
    a.seqs = ws.seqs;
    a.n_seq = m->ms_n_seq;
    a.n_rg = m->ms_n_rg;
    a.n_pg = m->ms_n_pg;
    a.pv_part = nullptr;
  }
  if (m->ctx->attn_fused && ws.fz_part) {
    a.fz_count = ws.fz_count;
    a.fz_ticket = ws.fz_ticket;
    a.fz_part = ws.fz_part;
    a.err = ws.err;
  }
  if (m->ctx->attn_decode && attn_decode_ok(a)) {
    // single-row decode: scores, statistics and P.V in one kernel (bit-identical)
    ALM_LAUNCH(launch_attn_decode(a, pdl, st));
    prof_mark(ALM_OP_ATTN, M);
  } else if (attn_fused_ok(a)) {
    ALM_LAUNCH(launch_attn_fused(a, pdl, st));
    prof_mark(ALM_OP_ATTN, M);
  } else {
    ALM_LAUNCH(launch_attention(a, pdl, st));
    prof_mark(ALM_OP_ATTN_PV, M);
  }

  if (m->tp) {
    // row-split O: fp32 partials, sum over ranks, then residual and norm partials
    ALM_TRY(enqueue_tp_rowsplit(m, L.o, raw_in(ws.ctx, qdim, qdim), M, in, ws.s1, ws.ss1, pdl));
    prof_mark(ALM_OP_O, M);
  } else {
    Epi eo;
    eo.out = ws.s1;
    eo.ldo = c.hidden;
    eo.n_out = c.hidden;
    eo.res = in;
    eo.ss_out = ws.ss1;
    ALM_LAUNCH(launch_gemv(L.o->t, raw_in(ws.ctx, qdim, qdim), M, EPI_RESID, eo, io, scr, pdl, st));
    prof_mark(ALM_OP_O, M);
  }

  const ActIn n1 = deferred_in(m, ws.s1, ws.ss1, L.n_in);
  Epi eg;
  eg.out = ws.h;
  eg.ldo = c.intermediate;
  eg.n_out = c.intermediate;
  ALM_LAUNCH(launch_gemv(L.gu->t, n1, M, EPI_SWIGLU, eg, io, scr, pdl, st));
  prof_mark(ALM_OP_GATE_UP, M);

  if (m->tp) {
    ALM_TRY(enqueue_tp_rowsplit(m, L.down, raw_in(ws.h, c.intermediate, c.intermediate), M, n1, ws.s2, ws.ss2, pdl));
    prof_mark(ALM_OP_DOWN, M);
    return ALM_OK;
  }
  Epi ed;
  ed.out = ws.s2;
  ed.ldo = c.hidden;
  ed.n_out = c.hidden;
  ed.res = n1;
  ed.ss_out = ws.ss2;
  ALM_LAUNCH(launch_gemv(L.down->t, raw_in(ws.h, c.intermediate, c.intermediate), M, EPI_RESID, ed, io, scr,
                         pdl, st));
  prof_mark(ALM_OP_DOWN, M);
  return ALM_OK;
}

// Head on normalised rows `x` (M, hidden) already in ws.xn.
int enqueue_head_tp(alm_model* m, int M, bool pdl) {
  Work& ws = m->ws;
  cudaStream_t st = m->ctx->stream;
  const int world = m->ctx->tp_world;
  Epi e;
  e.out = ws.logits_local;
  e.ldo = m->vocab_local;
  e.n_out = m->vocab_local;
  e.am_val = ws.am_val;
  e.am_idx = ws.am_idx;
  const ActIn in = raw_in(ws.xn, m->cfg.hidden, m->cfg.hidden);
  ALM_LAUNCH(launch_gemv(m->head->t, in, M, EPI_LOGITS, e, StepIO{ws.pos, ws.err}, scratch_of(m), pdl, st));
  prof_mark(ALM_OP_HEAD, M);
  // (value, global index) of each rank's best, gathered; the best of them
  int* send = ws.tp_pairs;
  int* recv = ws.tp_pairs + 2 * kMaxRows;
  ALM_LAUNCH(launch_tp_argmax_local(ws.am_val, ws.am_idx, ws.n_am, M, m->vocab_offset, send, pdl, st));
  std::string err;
  if (tp_allgather(m->ctx->tp_comm, send, recv, static_cast<size_t>(M) * 2 * sizeof(int), st, &err))
    return fail(ALM_ERR_CUDA, err);
  ALM_LAUNCH(launch_tp_argmax_pick(recv, world, M, ws.argmax, false, st));
  prof_mark(ALM_OP_ARGMAX, M);
  if (m->tp_need_logits) {
    if (tp_allgather(m->ctx->tp_comm, ws.logits_local, ws.logits_gather,
                     static_cast<size_t>(M) * m->vocab_local * sizeof(half), st, &err))
      return fail(ALM_ERR_CUDA, err);
    ALM_LAUNCH(launch_tp_logits_reorder(ws.logits_gather, world, M, m->vocab_local, ws.logits, false, st));
  }
  return ALM_OK;
}

int enqueue_head(alm_model* m, int M, bool pdl) {
  if (m->tp) return enqueue_head_tp(m, M, pdl);
  Work& ws = m->ws;
  Epi e;
  e.out = ws.logits;
  e.ldo = m->cfg.vocab;
  e.n_out = m->cfg.vocab;
  e.am_val = ws.am_val;
  e.am_idx = ws.am_idx;
  const ActIn in = raw_in(ws.xn, m->cfg.hidden, m->cfg.hidden);
  ALM_LAUNCH(launch_gemv(m->head->t, in, M, EPI_LOGITS, e, StepIO{ws.pos, ws.err}, scratch_of(m), pdl, m->ctx->stream));
  prof_mark(ALM_OP_HEAD, M);
  ALM_LAUNCH(launch_argmax_final(ws.am_val, ws.am_idx, ws.n_am, M, ws.argmax, pdl, m->ctx->stream));
  prof_mark(ALM_OP_ARGMAX, M);
  return ALM_OK;
}

EmbedArgs embed_args(alm_model* m, int M) {
  Work& ws = m->ws;
  EmbedArgs ea;
  ea.table = m->embed_table;
  ea.scale = m->embed_scale;
  ea.bits = m->embed_bits;
  ea.block = m->embed_block;
  ea.nsb = m->embed_nsb;
  ea.hidden = m->cfg.hidden;
  ea.row_bytes = m->embed_row_bytes;
  ea.vocab = m->cfg.vocab;
  ea.tokens = ws.tokens;
  ea.out = ws.x0;
  ea.M = M;
  ea.err = ws.err;
  return ea;
}

// Device layer table, barrier counter and launch shape of the persistent
// forward kernel (fwd_grid stays 0 when the kernel cannot keep all its CTAs
// resident, and forwards then use the standalone kernels).
int build_forward(alm_model* m) {
  const alm_model_config& c = m->cfg;
  m->fwd_grid = 0;
  // a model may be finalized before its layers are set (the drop-in
  // LlamaModel uploads each layer dict on first use): no persistent kernel
  // until every layer is present
  for (const Layer& L : m->layers)
    if (!L.qkv) return ALM_OK;
  std::vector<FwdLayer> host(c.layers);
  size_t stage = gemv_stage_bytes(m->head->t, kPersistRows);
  for (int li = 0; li < c.layers; ++li) {
    const Layer& L = m->layers[li];
    host[li].qkv = L.qkv->t;
    host[li].o = L.o->t;
    host[li].gu = L.gu->t;
    host[li].down = L.down->t;
    host[li].n_in = L.n_in;
    host[li].n_post = L.n_post;
    for (const alm_qweight* w : {L.qkv, L.o, L.gu, L.down}) stage = std::max(stage, gemv_stage_bytes(w->t, kPersistRows));
  }
  if (!m->fwd_layers) ALM_TRY(dev_alloc_t(&m->fwd_layers, static_cast<size_t>(c.layers)));
  ALM_CUDA(cudaMemcpy(m->fwd_layers, host.data(), host.size() * sizeof(FwdLayer), cudaMemcpyHostToDevice));
  if (!m->fwd_bar) {
    ALM_TRY(dev_alloc_t(&m->fwd_bar, 1));
    ALM_CUDA(cudaMemset(m->fwd_bar, 0, sizeof(unsigned long long)));
  }
  m->fwd_grid = 0;
  m->fwd_smem = forward_smem_bytes(stage, c.head_dim, c.hidden);
  // the persistent kernel runs the tile-layout GEMV with 64-column scale blocks only
  auto persistable = [](const alm_qweight* w) { return w->t.layout == kLayoutTile && w->t.sb != 2; };
  if (!persistable(m->head)) return ALM_OK;
  for (const Layer& L : m->layers)
    for (const alm_qweight* w : {L.qkv, L.o, L.gu, L.down})
      if (!persistable(w)) return ALM_OK;
  if (forward_barriers(c.layers, true) > kBarRound || c.head_dim % 16 || c.head_dim > 256) return ALM_OK;
  int per_sm = 0;
  if (forward_init_attrs(m->fwd_smem, &per_sm) != cudaSuccess) {
    cudaGetLastError();
    return ALM_OK;
  }
  if (per_sm >= 1) m->fwd_grid = m->ctx->n_sms * std::min(per_sm, 2);
  return ALM_OK;
}

FwdParams forward_params(alm_model* m, alm_kv* kv, int M, bool head) {
  const alm_model_config& c = m->cfg;
  Work& ws = m->ws;
  FwdParams p;
  p.layers = m->fwd_layers;
  p.n_layers = c.layers;
  p.M = M;
  p.hidden = c.hidden;
  p.inter = c.intermediate;
  p.heads = c.heads;
  p.kv_heads = c.kv_heads;
  p.head_dim = c.head_dim;
  p.vocab = c.vocab;
  p.eps = c.rms_eps;
  p.sqrt_hd = static_cast<float>(sqrt(static_cast<double>(c.head_dim)));
  p.embed = embed_args(m, M);
  p.s1 = ws.s1;
  p.s2 = ws.s2;
  p.ss1 = ws.ss1;
  p.ss2 = ws.ss2;
  p.q = ws.q;
  p.ctx = ws.ctx;
  p.h = ws.h;
  p.xn = ws.xn;
  p.logits = ws.logits;
  p.part = ws.part;
  p.kcache = kv->k;
  p.vcache = kv->v;
  p.kv_layer_elems = kv->layer_elems;
  p.page_table = kv->page_table;
  p.page_size = kv->page_size;
  p.max_ctx = kv->max_len;
  p.scores = ws.scores;
  p.score_ld = ws.score_ld;
  p.stats = ws.stats;
  p.rope = m->rope;
  p.do_head = head ? 1 : 0;
  p.head = m->head->t;
  p.final_norm = m->final_norm;
  p.am_val = ws.am_val;
  p.am_idx = ws.am_idx;
  p.argmax = ws.argmax;
  p.io = StepIO{ws.pos, ws.err};
  p.bar = m->fwd_bar;
  return p;
}

int enqueue_forward_persistent(alm_model* m, alm_kv* kv, int M, bool head,
                               unsigned long long* trace = nullptr) {
  FwdParams p = forward_params(m, kv, M, head);
  p.trace = trace;
  ALM_LAUNCH(launch_forward(p, m->fwd_grid, m->fwd_smem, m->ctx->stream));
  return ALM_OK;
}

// Whether the model's single-row forwards can run as the cluster kernel, and
// its shared memory.  Needs the device layer table of build_forward.
int build_cluster_fwd(alm_model* m) {
  m->cf_ok = false;
  if (!m->fwd_layers) return ALM_OK;
  const alm_model_config& c = m->cfg;
  if (c.head_dim % 16 || c.head_dim > 256 || c.heads % c.kv_heads) return ALM_OK;
  int max_kb = 0;
  for (const Layer& L : m->layers) {
    if (!L.qkv) return ALM_OK;
    for (const alm_qweight* w : {L.qkv, L.o, L.gu, L.down}) {
      if (!cluster_fwd_weight_ok(w->t)) return ALM_OK;
      max_kb = std::max(max_kb, w->t.k_blocks);
    }
  }
  const size_t smem = cluster_fwd_smem_bytes(max_kb, c.head_dim);
  if (smem > 227 * 1024 - 16 * 1024) return ALM_OK;   // static shared memory stays below the rest
  int n_clusters = 0;
  if (cluster_fwd_init(smem, &n_clusters) != cudaSuccess) {
    cudaGetLastError();
    return ALM_OK;
  }
  if (n_clusters < 1) return ALM_OK;
  m->cf_smem = smem;
  m->cf_ok = true;
  return ALM_OK;
}

// Embedding (tokens already in ws.tokens, position in ws.pos) -> all layers ->
// final norms -> head.
int enqueue_forward(alm_model* m, alm_kv* kv, int M, bool head, bool pdl) {
  if (m->ctx->persist && m->fwd_grid > 0 && M <= kPersistRows && m->ms_n_seq == 0)
    return enqueue_forward_persistent(m, kv, M, head);
  Work& ws = m->ws;
  if (M == 1 && m->ctx->cluster && m->cf_ok && m->ms_n_seq == 0) {
    // embedding and every layer in one cluster launch, then the final norm
    // and the head over the whole GPU
    ALM_LAUNCH(launch_cluster_fwd(forward_params(m, kv, 1, false), m->cf_smem, pdl, m->ctx->stream));
    prof_mark(ALM_OP_LAYERS, M);
    if (!head) return ALM_OK;
    const ActIn fin = deferred_in(m, ws.s2, ws.ss2, m->layers[m->cfg.layers - 1].n_post);
    ALM_LAUNCH(launch_rownorm(fin, M, m->final_norm, m->cfg.rms_eps, ws.xn, m->cfg.hidden, pdl, m->ctx->stream));
    prof_mark(ALM_OP_FINAL_NORM, M);
    return enqueue_head(m, M, pdl);
  }
  EmbedArgs ea;
  ea.table = m->embed_table;
  ea.scale = m->embed_scale;
  ea.bits = m->embed_bits;
  ea.block = m->embed_block;
  ea.nsb = m->embed_nsb;
  ea.hidden = m->cfg.hidden;
  ea.row_bytes = m->embed_row_bytes;
  ea.vocab = m->cfg.vocab;
  ea.tokens = ws.tokens;
  ea.out = ws.x0;
  ea.M = M;
  ea.err = ws.err;
  ALM_LAUNCH(launch_embed(ea, pdl, m->ctx->stream));
  prof_mark(ALM_OP_EMBED, M);
  ActIn in = raw_in(ws.x0, m->cfg.hidden, m->cfg.hidden);
  for (int li = 0; li < m->cfg.layers; ++li) {
    ALM_TRY(enqueue_layer(m, li, kv, M, in, pdl));
    in = deferred_in(m, ws.s2, ws.ss2, m->layers[li].n_post);
  }
  if (!head) return ALM_OK;
  ALM_LAUNCH(launch_rownorm(in, M, m->final_norm, m->cfg.rms_eps, ws.xn, m->cfg.hidden, pdl, m->ctx->stream));
  prof_mark(ALM_OP_FINAL_NORM, M);
  return enqueue_head(m, M, pdl);
}

// ---- batched prefill through the dense path ----------------------------------
// Buffers of a prefill chunk (kMaxDenseRows rows) and the attention scratch for
// contexts of up to max_ctx positions.
int ensure_prefill(alm_model* m, int max_ctx) {
  const alm_model_config& c = m->cfg;
  PrefillWork& pf = m->pf;
  const int R = kMaxDenseRows, H = c.hidden, qd = c.heads * c.head_dim, kd = c.kv_heads * c.head_dim;
  const int I = c.intermediate;
  auto r8 = [](int v) { return (v + 7) / 8 * 8; };   // 16-byte row strides for the tensor-map loads
  if (pf.rows == 0) {
    pf.ld_qkv = r8(qd + 2 * kd);
    pf.ld_gu = r8(2 * I);
    pf.ld_h = r8(I);
    // split-K partials of any chunk size the dense path takes (17..R rows)
    size_t part = 0;
    for (const DenseLayer& D : m->dense)
      for (const alm_qweight* w : {D.qkv, D.o, D.gu, D.down})
        if (w)
          for (int rows = kMaxRows + 1; rows <= R; ++rows) part = std::max(part, tc_part_floats(w->t, rows));
    int rc = dev_alloc_t(&pf.tokens, R);
    if (rc == ALM_OK) rc = dev_alloc_t(&pf.xa, static_cast<size_t>(R) * H);
    if (rc == ALM_OK) rc = dev_alloc_t(&pf.xb, static_cast<size_t>(R) * H);
    if (rc == ALM_OK) rc = dev_alloc_t(&pf.qkv, static_cast<size_t>(R) * pf.ld_qkv);
    if (rc == ALM_OK) rc = dev_alloc_t(&pf.q, static_cast<size_t>(R) * qd);
    if (rc == ALM_OK) rc = dev_alloc_t(&pf.ctx, static_cast<size_t>(R) * qd);
    if (rc == ALM_OK) rc = dev_alloc_t(&pf.o, static_cast<size_t>(R) * H);
    if (rc == ALM_OK) rc = dev_alloc_t(&pf.s, static_cast<size_t>(R) * H);
    if (rc == ALM_OK) rc = dev_alloc_t(&pf.ss, static_cast<size_t>(R) * n_h_tiles(m));
    if (rc == ALM_OK) rc = dev_alloc_t(&pf.gu, static_cast<size_t>(R) * pf.ld_gu);
    if (rc == ALM_OK) rc = dev_alloc_t(&pf.h, static_cast<size_t>(R) * pf.ld_h);
    if (rc == ALM_OK && part) rc = dev_alloc_t(&pf.part, part);
    if (rc != ALM_OK) {
      free_prefill_work(pf);
      return rc;
    }
    pf.part_floats = part;
    pf.rows = R;
  }
  if (max_ctx > pf.attn_ctx) {
    dev_free(pf.scores);
    dev_free(pf.stats);
    pf.scores = nullptr;
    pf.stats = nullptr;
    pf.attn_ctx = 0;
    const int gq = c.heads / c.kv_heads;
    const int n_rg = (R * gq + kAttnRows - 1) / kAttnRows;
    const int cap = (max_ctx + kAttnChunk - 1) / kAttnChunk * kAttnChunk;
    const int ld = cap + kAttnChunk;   // the P.V pass reads whole 16-position groups
    ALM_TRY(dev_alloc_t(&pf.scores, static_cast<size_t>(c.kv_heads) * n_rg * kAttnRows * ld));
    ALM_TRY(dev_alloc_t(&pf.stats, static_cast<size_t>(c.kv_heads) * n_rg * (cap / kAttnChunk) * kAttnRows * 2));
    pf.attn_ctx = cap;
    pf.score_ld = ld;
  }
  return ALM_OK;
}

// One prefill chunk of M (17..256) rows at positions pos0.. (tokens already
// in pf.tokens, ws.pos = pos0): every projection through the dense tcgen05
// path, the fused epilogues' operations in row kernels, the attention passes
// over the chunk's rows.  Only the KV cache is kept; the last layer stops
// after its KV write.  The arithmetic is the M <= 16 path's, so the cache
// equals a 16-row-chunk prefill up to the matmuls' fp32 summation order.
int enqueue_prefill_dense(alm_model* m, alm_kv* kv, int M, int pos0, int slot) {
  const alm_model_config& c = m->cfg;
  PrefillWork& pf = m->pf;
  Work& ws = m->ws;
  cudaStream_t st = m->ctx->stream;
  const bool pdl = m->ctx->pdl;
  const int H = c.hidden, hd = c.head_dim, qd = c.heads * hd, I = c.intermediate;
  const StepIO io{ws.pos, ws.err};
  const SplitScratch scr{pf.part, pf.part_floats};
  auto dense = [&](const alm_qweight* w, const half* x, int ldx, half* y, int ldy) -> int {
    Epi e;
    e.out = y;
    e.ldo = ldy;
    e.n_out = w->out;
    ALM_LAUNCH(launch_gemv(w->t, raw_in(x, ldx, w->in_real), M, EPI_STORE, e, io, scr, pdl, st));
    return ALM_OK;
  };
  EmbedArgs ea;
  ea.table = m->embed_table;
  ea.scale = m->embed_scale;
  ea.bits = m->embed_bits;
  ea.block = m->embed_block;
  ea.nsb = m->embed_nsb;
  ea.hidden = H;
  ea.row_bytes = m->embed_row_bytes;
  ea.vocab = c.vocab;
  ea.tokens = pf.tokens;
  ea.out = pf.xa;
  ea.M = M;
  ea.err = ws.err;
  ALM_LAUNCH(launch_embed(ea, pdl, st));
  for (int li = 0; li < c.layers; ++li) {
    const Layer& L = m->layers[li];
    const DenseLayer& D = m->dense[li];
    // the input of a layer after the first: the previous layer's output under
    // its n_post norm, written into xa by that layer's last residual kernel
    ALM_TRY(dense(D.qkv, pf.xa, H, pf.qkv, pf.ld_qkv));
    PfRopeArgs ra;
    ra.qkv = pf.qkv;
    ra.ld_qkv = pf.ld_qkv;
    ra.rope = m->rope;
    ra.pos0 = pos0;
    ra.heads = c.heads;
    ra.kv_heads = c.kv_heads;
    ra.head_dim = hd;
    ra.q = pf.q;
    ra.ldq = qd;
    ra.kcache = kv->k + static_cast<size_t>(li) * kv->layer_elems;
    ra.vcache = kv->v + static_cast<size_t>(li) * kv->layer_elems;
    ra.page_table = kv->page_table + static_cast<size_t>(slot) * kv->pages_per_slot;
    ra.page_size = kv->page_size;
    ALM_LAUNCH(launch_pf_rope_kv(ra, M, pdl, st));
    AttnArgs a;
    a.q = pf.q;
    a.ldq = qd;
    a.kcache = ra.kcache;
    a.vcache = ra.vcache;
    a.page_table = ra.page_table;
    a.page_size = kv->page_size;
    a.heads = c.heads;
    a.kv_heads = c.kv_heads;
    a.head_dim = hd;
    a.M = M;
    a.pos = ws.pos;
    a.max_ctx = pos0 + M;   // exact: the host knows this chunk's context
    a.scores = pf.scores;
    a.score_ld = pf.score_ld;
    a.stats = pf.stats;
    a.ctx = pf.ctx;
    a.ldc = qd;
    ALM_LAUNCH(launch_attention_prefill(a, pdl, st));
    if (li == c.layers - 1) break;
    ALM_TRY(dense(D.o, pf.ctx, qd, pf.o, H));
    ALM_LAUNCH(launch_resid_norm(raw_in(pf.xa, H, H), pf.o, M, H, pf.s, pf.ss, deferred_in(m, pf.s, pf.ss, L.n_in),
                                 pf.xb, H, pdl, st));
    ALM_TRY(dense(D.gu, pf.xb, H, pf.gu, pf.ld_gu));
    ALM_LAUNCH(launch_pf_swiglu(pf.gu, pf.ld_gu, I, M, pf.h, pf.ld_h, pdl, st));
    ALM_TRY(dense(D.down, pf.h, pf.ld_h, pf.o, H));
    ALM_LAUNCH(launch_resid_norm(raw_in(pf.xb, H, H), pf.o, M, H, pf.s, pf.ss, deferred_in(m, pf.s, pf.ss, L.n_post),
                                 pf.xa, H, pdl, st));
  }
  return ALM_OK;
}

// Sampler arguments for rows of a model's last logits, writing the picks
// into its argmax buffer.
SampleArgs sample_args(alm_model* m, float temperature, float top_p, float min_p, const double* uniforms,
                       const int* cursor, int offset) {
  SampleArgs a;
  a.logits = m->ws.logits;
  a.ld = m->cfg.vocab;
  a.vocab = m->cfg.vocab;
  a.temperature = temperature;
  a.top_p = top_p;
  a.min_p = min_p;
  a.uniforms = uniforms;
  a.u_cursor = cursor;
  a.u_offset = offset;
  a.scratch = m->ws.sample_scratch;
  a.out = m->ws.argmax;
  return a;
}

int ensure_sample_scratch(alm_model* m) {
  if (!m->ws.sample_scratch)
    ALM_TRY(dev_alloc_t(&m->ws.sample_scratch, static_cast<size_t>(kMaxPassRows) * m->cfg.vocab));
  return ALM_OK;
}

int check_ready(alm_model* m) {
  ALM_REQ(m != nullptr, "null model");
  if (!m->finalized) return fail(ALM_ERR_STATE, "model not finalized");
  return ALM_OK;
}

int check_layers(alm_model* m) {
  for (int i = 0; i < m->cfg.layers; ++i)
    if (!m->layers[i].qkv) return fail(ALM_ERR_STATE, "layer " + std::to_string(i) + " not set");
  return ALM_OK;
}

int check_kv(alm_model* m, alm_kv* kv, int rows, int pos0) {
  ALM_REQ(kv != nullptr, "null kv");
  ALM_REQ(kv->n_layers == m->cfg.layers && kv->kv_heads == m->cfg.kv_heads && kv->head_dim == m->cfg.head_dim,
          "kv cache shape mismatch");
  ALM_REQ(rows >= 1 && rows <= kMaxRows, "rows must be in 1..16");
  ALM_REQ(pos0 >= 0 && pos0 + rows <= kv->max_len, "pos out of kv cache range");
  ALM_REQ(pos0 + rows <= m->cfg.max_len, "pos out of rope table range");
  return ensure_attn(m, kv->max_len);
}

int sync_and_check(alm_model* m) {
  ALM_CUDA(cudaStreamSynchronize(m->ctx->stream));
  int err = 0;
  ALM_CUDA(cudaMemcpy(&err, m->ws.err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) {
    cudaMemset(m->ws.err, 0, sizeof(int));
    if (err == 2) return fail(ALM_ERR_CUDA, "a device-side wait gave up (weight stream did not arrive)");
    if (err == 3) return fail(ALM_ERR_CUDA, "a device-side wait gave up (grid barrier of the persistent forward)");
    if (err == 4) return fail(ALM_ERR_CUDA, "a device-side wait gave up (cluster forward)");
    return fail(ALM_ERR_TOKEN, "token id outside the vocabulary");
  }
  return ALM_OK;
}

int set_pos(alm_model* m, int pos0) {
  m->ws.pinned[0] = pos0;
  ALM_CUDA(cudaMemcpyAsync(m->ws.pos, m->ws.pinned, sizeof(int), cudaMemcpyHostToDevice, m->ctx->stream));
  ALM_CUDA(cudaStreamSynchronize(m->ctx->stream));
  return ALM_OK;
}

int copy_logits_out(alm_model* m, int rows, float* logits_host, int32_t* argmax_host) {
  cudaStream_t st = m->ctx->stream;
  if (logits_host) {
    std::vector<half> tmp(static_cast<size_t>(rows) * m->cfg.vocab);
    ALM_CUDA(cudaMemcpyAsync(tmp.data(), m->ws.logits, tmp.size() * sizeof(half), cudaMemcpyDeviceToHost, st));
    ALM_CUDA(cudaStreamSynchronize(st));
    for (size_t i = 0; i < tmp.size(); ++i) logits_host[i] = __half2float(tmp[i]);
  }
  if (argmax_host) {
    ALM_CUDA(cudaMemcpyAsync(argmax_host, m->ws.argmax, rows * sizeof(int), cudaMemcpyDeviceToHost, st));
    ALM_CUDA(cudaStreamSynchronize(st));
  }
  return ALM_OK;
}

}  // namespace

// ============================================================================
// C ABI
// ============================================================================
extern "C" {

const char* alm_last_error(void) { return g_err.c_str(); }
int alm_abi_version(void) { return 100; }

int alm_ctx_create(int device, alm_ctx** out) {
  ALM_REQ(out != nullptr, "null out");
  int n = 0;
  ALM_CUDA(cudaGetDeviceCount(&n));
  ALM_REQ(device >= 0 && device < n, "no such CUDA device");
  ALM_CUDA(cudaSetDevice(device));
  {
    cudaError_t e = gemv_init_attrs();
    if (e == cudaSuccess) e = attention_init_attrs();
    if (e == cudaSuccess) e = attn_decode_init_attrs();
    if (e == cudaSuccess) e = attn_prefill_init_attrs();
    if (e == cudaSuccess) e = rows_init_attrs();
    if (e == cudaSuccess) e = sample_init_attrs();
    if (e != cudaSuccess) return fail(ALM_ERR_CUDA, std::string("kernel attributes: ") + cudaGetErrorString(e));
  }
  auto* c = new alm_ctx();
  c->device = device;
  c->n_sms = n_sms_of(device);
  {
    const cudaError_t e = attn_fused_init_attrs(c->n_sms);
    if (e != cudaSuccess) {
      delete c;
      return fail(ALM_ERR_CUDA, std::string("kernel attributes: ") + cudaGetErrorString(e));
    }
  }
  {
    const char* e = getenv("ALM_NO_PDL");
    c->pdl = !(e && e[0] == '1');
    const char* e2 = getenv("ALM_PERSIST");
    c->persist = e2 && e2[0] == '1';
    const char* e5 = getenv("ALM_ATTN_DECODE");
    c->attn_decode = e5 && e5[0] == '1';
    const char* e4 = getenv("ALM_CLUSTER");
    c->cluster = e4 && e4[0] == '1';
    const char* e3 = getenv("ALM_TC");
    if (e3 && (e3[0] == '0' || e3[0] == '1' || e3[0] == '2')) c->tc = e3[0] - '0';
    const char* e6 = getenv("ALM_DENSE_PREFILL");
    c->dense_prefill = !(e6 && e6[0] == '0');
    const char* e7 = getenv("ALM_ATTN_FUSED");
    c->attn_fused = e7 && e7[0] == '1';
  }
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete c;
    return fail(ALM_ERR_CUDA, "stream creation failed");
  }
  *out = c;
  return ALM_OK;
}

int alm_ctx_destroy(alm_ctx* ctx) {
  if (!ctx) return ALM_OK;
  DeviceGuard g(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->p2p_ready)
    for (int r = 0; r < ctx->p2p.world; ++r)
      if (r != ctx->p2p.rank && ctx->p2p.areas[r]) cudaIpcCloseMemHandle(ctx->p2p.areas[r]);
  dev_free(ctx->p2p_own);
  dev_free(ctx->p2p.counters);
  tp_comm_destroy(ctx->tp_comm);
  cudaStreamDestroy(ctx->stream);
  delete ctx;
  return ALM_OK;
}

int alm_nccl_unique_id(uint8_t* id_out) {
  ALM_REQ(id_out, "null argument");
  std::string err;
  if (tp_unique_id(id_out, &err)) return fail(ALM_ERR_STATE, err);
  return ALM_OK;
}

int alm_ctx_init_tp(alm_ctx* ctx, int rank, int world, const uint8_t* id) {
  ALM_REQ(ctx && id, "null argument");
  ALM_REQ(world >= 1 && rank >= 0 && rank < world, "rank must be in 0..world-1");
  ALM_REQ(!ctx->tp_comm, "tensor parallelism already initialised on this context");
  DeviceGuard g(ctx->device);
  std::string err;
  void* comm = nullptr;
  if (tp_comm_init(rank, world, id, &comm, &err)) return fail(ALM_ERR_STATE, err);
  ctx->tp_comm = comm;
  ctx->tp_rank = rank;
  ctx->tp_world = world;
  return ALM_OK;
}

int alm_tp_p2p_open(alm_ctx* ctx, int row_floats, uint8_t* handle_out) {
  ALM_REQ(ctx && handle_out, "null argument");
  ALM_REQ(ctx->tp_comm && ctx->tp_world >= 2 && ctx->tp_world <= kTpP2pMaxWorld,
          "peer all-reduce needs a tensor-parallel context of 2..8 ranks");
  ALM_REQ(row_floats > 0 && row_floats % 4 == 0, "row_floats must be a positive multiple of 4");
  ALM_REQ(!ctx->p2p_own, "peer all-reduce already opened");
  DeviceGuard g(ctx->device);
  TpP2p& p = ctx->p2p;
  p.world = ctx->tp_world;
  p.rank = ctx->tp_rank;
  p.rows = kMaxRows;
  p.row_floats = row_floats;
  const size_t bytes = tp_p2p_area_bytes(p.world, p.rows, p.row_floats);
  ALM_TRY(dev_alloc(reinterpret_cast<void**>(&ctx->p2p_own), bytes));
  ALM_CUDA(cudaMemset(ctx->p2p_own, 0, bytes));
  ALM_TRY(dev_alloc_t(&p.counters, kMaxRows));
  ALM_CUDA(cudaMemset(p.counters, 0, kMaxRows * sizeof(unsigned)));
  static_assert(sizeof(cudaIpcMemHandle_t) == kTpP2pHandleBytes, "IPC handle size");
  ALM_CUDA(cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle_out), ctx->p2p_own));
  return ALM_OK;
}

int alm_tp_p2p_connect(alm_ctx* ctx, const uint8_t* handles) {
  ALM_REQ(ctx && handles, "null argument");
  ALM_REQ(ctx->p2p_own && !ctx->p2p_ready, "open the peer all-reduce first (once)");
  DeviceGuard g(ctx->device);
  TpP2p& p = ctx->p2p;
  for (int r = 0; r < p.world; ++r) {
    if (r == p.rank) {
      p.areas[r] = ctx->p2p_own;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles + static_cast<size_t>(r) * kTpP2pHandleBytes, sizeof(h));
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != p.rank && p.areas[q]) cudaIpcCloseMemHandle(p.areas[q]);
      for (float*& a : p.areas) a = nullptr;
      return fail(ALM_ERR_CUDA, std::string("peer area of rank ") + std::to_string(r) + ": " + cudaGetErrorString(e));
    }
    p.areas[r] = static_cast<float*>(ptr);
  }
  // every rank's area is zeroed before any rank sends: the caller connects
  // all ranks before the first forward
  ctx->p2p_ready = true;
  ctx->tp_p2p = true;
  return ALM_OK;
}

int alm_ctx_set_tp_p2p(alm_ctx* ctx, int enable) {
  ALM_REQ(ctx, "null context");
  ALM_REQ(!enable || ctx->p2p_ready, "the peer all-reduce is not connected");
  ctx->tp_p2p = enable != 0;
  return ALM_OK;
}

int alm_ctx_set_persistent(alm_ctx* ctx, int enable) {
  ALM_REQ(ctx, "null context");
  ctx->persist = enable != 0;
  return ALM_OK;
}

int alm_ctx_set_attn_fused(alm_ctx* ctx, int enable) {
  ALM_REQ(ctx, "null context");
  ctx->attn_fused = enable != 0;
  return ALM_OK;
}

int alm_ctx_set_cluster_forward(alm_ctx* ctx, int enable) {
  ALM_REQ(ctx, "null context");
  ctx->cluster = enable != 0;
  return ALM_OK;
}

int alm_model_cluster_forward(const alm_model* m, int* uses_cluster) {
  ALM_REQ(m && uses_cluster, "null argument");
  *uses_cluster = (m->cf_ok && m->ctx->cluster) ? 1 : 0;
  return ALM_OK;
}

int alm_ctx_set_gemv_layout(alm_ctx* ctx, int mode) {
  ALM_REQ(ctx, "null context");
  ALM_REQ(mode >= 0 && mode <= 2, "mode must be 0 (tile layout), 1 (row layout for large weights) or 2 (row layout)");
  ctx->tc = mode;
  return ALM_OK;
}

int alm_ctx_sync(alm_ctx* ctx) {
  ALM_REQ(ctx, "null ctx");
  DeviceGuard g(ctx->device);
  ALM_CUDA(cudaStreamSynchronize(ctx->stream));
  return ALM_OK;
}

int alm_dev_alloc(alm_ctx* ctx, size_t bytes, void** out_dev) {
  ALM_REQ(ctx && out_dev, "null argument");
  DeviceGuard g(ctx->device);
  return dev_alloc(out_dev, bytes);
}
int alm_dev_free(alm_ctx* ctx, void* dev) {
  ALM_REQ(ctx, "null ctx");
  DeviceGuard g(ctx->device);
  ALM_CUDA(cudaFree(dev));
  return ALM_OK;
}
int alm_copy_h2d(alm_ctx* ctx, void* dst_dev, const void* src_host, size_t bytes) {
  ALM_REQ(ctx && dst_dev && src_host, "null argument");
  DeviceGuard g(ctx->device);
  ALM_CUDA(cudaMemcpyAsync(dst_dev, src_host, bytes, cudaMemcpyHostToDevice, ctx->stream));
  ALM_CUDA(cudaStreamSynchronize(ctx->stream));
  return ALM_OK;
}
int alm_copy_d2h(alm_ctx* ctx, void* dst_host, const void* src_dev, size_t bytes) {
  ALM_REQ(ctx && dst_host && src_dev, "null argument");
  DeviceGuard g(ctx->device);
  ALM_CUDA(cudaMemcpyAsync(dst_host, src_dev, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  ALM_CUDA(cudaStreamSynchronize(ctx->stream));
  return ALM_OK;
}

// ---- weights -----------------------------------------------------------------
int alm_qweight_upload(alm_ctx* ctx, const void* packed_host, const void* scale_host, int bits, int block,
                       int out, int in, int in_real, alm_qweight** w) {
  ALM_REQ(ctx && w, "null argument");
  ALM_REQ(out > 0, "out must be positive");
  DeviceGuard g(ctx->device);
  alm_proj_src s{packed_host, scale_host, bits, block, out, in, in_real};
  return build_qweight(ctx, &s, 1, identity_map(out), out, true, w);
}

int alm_qweight_set_split(alm_qweight* w, int ksw, int ksg) {
  ALM_REQ(w, "null weight");
  DeviceGuard g(w->ctx->device);
  QTile t = w->t;
  int grid_x = 0;
  if (t.layout == kLayoutRow) {
    // row layout: ksw = decoding warpgroups per CTA
    ALM_REQ((ksw == 1 || ksw == 2 || ksw == 4) && ksg >= 1 && ksg <= t.k_blocks,
            "row layout: ksw (warpgroups) must be 1, 2 or 4 and ksg at most the number of 64-column blocks");
    set_split_rows(t, ksw, ksg);
    ALM_REQ(tc_gemv_smem_bytes(t, kMaxRows) <= kRowSmemBudget, "per-CTA activation staging would exceed shared memory");
    grid_x = t.n_rb;
  } else {
    ALM_REQ((ksw == 1 || ksw == 2 || ksw == 4 || ksw == 8) && ksg >= 1 && ksw * ksg <= t.k_blocks,
            "ksw must be 1, 2, 4 or 8 and ksw * ksg at most the number of 64-column blocks");
    set_split(t, ksw, ksg);
    ALM_REQ(t.ksw * t.kps <= 64, "per-CTA activation staging would exceed shared memory");
    grid_x = (t.n_tiles + 8 / t.ksw - 1) / (8 / t.ksw) * kMaxRowGroups;   // per row group
  }
  unsigned* counters = nullptr;
  ALM_TRY(dev_alloc_t(&counters, grid_x));
  ALM_CUDA(cudaMemset(counters, 0, grid_x * sizeof(unsigned)));
  dev_free(w->counters);
  w->counters = counters;
  t.counters = counters;
  w->t = t;
  return ALM_OK;
}

int alm_qweight_get_split(const alm_qweight* w, int* ksw, int* ksg, int* kps) {
  ALM_REQ(w && ksw && ksg && kps, "null argument");
  *ksw = w->t.layout == kLayoutRow ? w->t.wg : w->t.ksw;
  *ksg = w->t.ksg;
  *kps = w->t.kps;
  return ALM_OK;
}

int alm_qweight_free(alm_qweight* w) {
  if (!w) return ALM_OK;
  DeviceGuard g(w->ctx->device);
  dev_free(w->data);
  dev_free(w->counters);
  delete w;
  return ALM_OK;
}

int alm_qweight_dequant(alm_ctx* ctx, const alm_qweight* w, uint16_t* out_host) {
  ALM_REQ(ctx && w && out_host, "null argument");
  DeviceGuard g(ctx->device);
  half* d = nullptr;
  const size_t n = static_cast<size_t>(w->out) * w->in_real;
  ALM_TRY(dev_alloc_t(&d, n));
  cudaError_t e = w->t.layout == kLayoutRow ? launch_dequant_rows(w->t, d, ctx->stream)
                                             : launch_dequant(w->t, d, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out_host, d, n * sizeof(half), cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  cudaFree(d);
  if (e != cudaSuccess) return fail(ALM_ERR_CUDA, std::string("dequant: ") + cudaGetErrorString(e));
  return ALM_OK;
}

int alm_qmatmul(alm_ctx* ctx, const alm_qweight* w, const uint16_t* x_dev, int ldx, int m, uint16_t* y_dev,
                int ldy) {
  ALM_REQ(ctx && w && x_dev && y_dev, "null argument");
  ALM_REQ(m >= 1 && m <= (w->t.layout == kLayoutRow ? kMaxDenseRows : kMaxRows),
          "m must be in 1..16 (1..256 for a row-layout weight)");
  ALM_REQ(ldx >= w->in_real && ldy >= w->out, "leading dimension too small");
  DeviceGuard g(ctx->device);
  static thread_local std::vector<std::pair<alm_ctx*, std::pair<float*, size_t>>> scratch;
  SplitScratch scr;
  const size_t need = gemv_part_floats(w->t, m);
  if (need) {
    std::pair<float*, size_t>* slot = nullptr;
    for (auto& p : scratch)
      if (p.first == ctx) slot = &p.second;
    if (!slot) {
      scratch.push_back({ctx, {nullptr, 0}});
      slot = &scratch.back().second;
    }
    if (slot->second < need) {
      dev_free(slot->first);
      slot->first = nullptr;
      slot->second = 0;
      ALM_TRY(dev_alloc_t(&slot->first, need));
      slot->second = need;
    }
    scr.part = slot->first;
    scr.part_floats = slot->second;
  }
  Epi e;
  e.out = reinterpret_cast<half*>(y_dev);
  e.ldo = ldy;
  e.n_out = w->out;
  ActIn in = raw_in(reinterpret_cast<const half*>(x_dev), ldx, w->in_real);
  ALM_CUDA(launch_gemv(w->t, in, m, EPI_STORE, e, StepIO{}, scr, false, ctx->stream));
  ALM_CUDA(cudaStreamSynchronize(ctx->stream));
  return ALM_OK;
}

int alm_matmul_f16_f16(alm_ctx* ctx, const uint16_t* a_host, const uint16_t* b_host, uint16_t* out_host, int m,
                       int k, int n) {
  ALM_REQ(ctx && a_host && b_host && out_host, "null argument");
  ALM_REQ(m >= 1 && m <= kMaxRows && k > 0 && n > 0, "shape out of range (m in 1..16)");
  DeviceGuard g(ctx->device);
  alm_qweight* w = nullptr;
  ALM_TRY(alm_qweight_upload(ctx, b_host, nullptr, 16, 0, n, k, k, &w));
  uint16_t *x = nullptr, *y = nullptr;
  int rc = dev_alloc_t(&x, static_cast<size_t>(m) * k);
  if (rc == ALM_OK) rc = dev_alloc_t(&y, static_cast<size_t>(m) * n);
  if (rc == ALM_OK) rc = alm_copy_h2d(ctx, x, a_host, static_cast<size_t>(m) * k * 2);
  if (rc == ALM_OK) rc = alm_qmatmul(ctx, w, x, k, m, y, n);
  if (rc == ALM_OK) rc = alm_copy_d2h(ctx, out_host, y, static_cast<size_t>(m) * n * 2);
  dev_free(x);
  dev_free(y);
  alm_qweight_free(w);
  return rc;
}

// ---- model -------------------------------------------------------------------
int alm_model_create(alm_ctx* ctx, const alm_model_config* cfg, const uint16_t* rope_host, alm_model** out) {
  ALM_REQ(ctx && cfg && rope_host && out, "null argument");
  const alm_model_config& c = *cfg;
  ALM_REQ(c.hidden > 0 && c.layers > 0 && c.heads > 0 && c.kv_heads > 0 && c.vocab > 0 && c.intermediate > 0,
          "invalid config");
  ALM_REQ(c.heads % c.kv_heads == 0, "heads must be a multiple of kv_heads");
  ALM_REQ(c.head_dim % 16 == 0 && c.head_dim <= 256, "head_dim must be a multiple of 16, <= 256");
  ALM_REQ(c.intermediate % 8 == 0, "intermediate must be a multiple of 8");
  ALM_REQ(c.max_len > 0, "invalid max_len");
  DeviceGuard g(ctx->device);
  auto* m = new alm_model();
  m->ctx = ctx;
  m->cfg = c;
  m->layers.resize(c.layers);
  m->dense.resize(c.layers);
  const size_t n = static_cast<size_t>(c.max_len) * c.head_dim;
  int rc = dev_alloc_t(&m->rope, n);
  if (rc == ALM_OK && cudaMemcpy(m->rope, rope_host, n * sizeof(half), cudaMemcpyHostToDevice) != cudaSuccess)
    rc = fail(ALM_ERR_CUDA, "rope upload failed");
  if (rc != ALM_OK) {
    alm_model_destroy(m);
    return rc;
  }
  *out = m;
  return ALM_OK;
}

int alm_model_destroy(alm_model* m) {
  if (!m) return ALM_OK;
  DeviceGuard g(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  for (Layer& L : m->layers) {
    alm_qweight_free(L.qkv);
    alm_qweight_free(L.o);
    alm_qweight_free(L.gu);
    alm_qweight_free(L.down);
    dev_free(L.n_in);
    dev_free(L.n_post);
  }
  for (DenseLayer& D : m->dense) free_dense(D);
  free_prefill_work(m->pf);
  for (auto& kvg : m->ms_graphs) cudaGraphExecDestroy(kvg.second);
  m->ms_graphs.clear();
  alm_qweight_free(m->head);
  dev_free(m->rope);
  dev_free(m->embed_table);
  dev_free(m->embed_scale);
  dev_free(m->final_norm);
  Work& w = m->ws;
  for (void* p : {(void*)w.tokens, (void*)w.pos, (void*)w.err, (void*)w.x0, (void*)w.s1, (void*)w.s2,
                  (void*)w.ss1, (void*)w.ss2, (void*)w.q, (void*)w.ctx, (void*)w.h, (void*)w.xn, (void*)w.xout,
                  (void*)w.logits, (void*)w.am_val, (void*)w.am_idx, (void*)w.argmax, (void*)w.part,
                  (void*)w.scores, (void*)w.stats, (void*)w.pv_part, (void*)w.pv_ticket,
                  (void*)w.fz_count, (void*)w.fz_ticket, (void*)w.fz_part,
                  (void*)w.sample_scratch, (void*)w.o32, (void*)w.tp_pairs,
                  (void*)w.logits_local, (void*)w.logits_gather, (void*)w.rows, (void*)w.seqs,
                  (void*)w.u_rows})
    dev_free(p);
  if (w.pinned) cudaFreeHost(w.pinned);
  if (w.seq_host) cudaFreeHost(w.seq_host);
  dev_free(m->fwd_layers);
  dev_free(m->fwd_bar);
  delete m;
  return ALM_OK;
}

int alm_model_set_layer(alm_model* m, int li, const alm_proj_src* p, const uint16_t* n_in_host,
                        const uint16_t* n_post_host) {
  ALM_REQ(m && p && n_in_host && n_post_host, "null argument");
  ALM_REQ(li >= 0 && li < m->cfg.layers, "layer index out of range");
  const alm_model_config& c = m->cfg;
  const int hd = c.head_dim, half_d = hd / 2;
  const int qd = c.heads * hd, kd = c.kv_heads * hd;
  ALM_REQ(p[0].out == qd && p[1].out == kd && p[2].out == kd, "q/k/v output sizes do not match the config");
  ALM_REQ(p[0].in_real == c.hidden && p[3].out == c.hidden && p[3].in_real == qd, "q/o sizes do not match");
  ALM_REQ(p[4].out == c.intermediate && p[5].out == c.intermediate && p[6].out == c.hidden &&
              p[6].in_real == c.intermediate && p[4].in_real == c.hidden,
          "gate/up/down sizes do not match");
  DeviceGuard g(m->ctx->device);
  Layer& L = m->layers[li];
  // fused QKV: q and k rows permuted so tile rows g / g+8 are RoPE pairs
  // (d, d + head_dim/2) of one head; v rows in order.
  std::vector<int> qkv_map(padded_rows(qd + 2 * kd, kLayoutTile), -1);
  auto rope_rows = [&](int src, int n_heads, int dst0) {
    for (int h = 0; h < n_heads; ++h)
      for (int d = 0; d < hd; ++d) {
        const int lo = d < half_d;
        const int dd = lo ? d : d - half_d;
        const int dst = dst0 + h * hd + (dd / 8) * 16 + (lo ? 0 : 8) + dd % 8;
        qkv_map[dst] = (src << 24) | (h * hd + d);
      }
  };
  rope_rows(0, c.heads, 0);
  rope_rows(1, c.kv_heads, qd);
  for (int r = 0; r < kd; ++r) qkv_map[qd + kd + r] = (2 << 24) | r;
  // fused gate/up, tile layout: tile rows g = gate j, g + 8 = up j (j = 8 * tile + g);
  // row layout: rows 0-15 of a 32-row group = gate j, rows 16-31 = up j (j = 16 * group + t)
  const int inter = c.intermediate;
  auto gu_map = [inter](int layout) {
    std::vector<int> mp(padded_rows(2 * inter, layout), -1);
    const int half_rows = layout == kLayoutRow ? 16 : 8;
    for (int j = 0; j < inter; ++j) {
      mp[(j / half_rows) * 2 * half_rows + j % half_rows] = (0 << 24) | j;
      mp[(j / half_rows) * 2 * half_rows + half_rows + j % half_rows] = (1 << 24) | j;
    }
    return mp;
  };
  alm_qweight *qkv = nullptr, *o = nullptr, *gu = nullptr, *dn = nullptr;
  const char* part = "qkv";
  int rc = build_qweight(m->ctx, &p[0], 3, [&qkv_map](int) { return qkv_map; }, qd + 2 * kd, false, &qkv);
  if (rc == ALM_OK) {
    part = "o";
    rc = build_qweight(m->ctx, &p[3], 1, identity_map(c.hidden), c.hidden, true, &o);
  }
  if (rc == ALM_OK) {
    part = "gate/up";
    rc = build_qweight(m->ctx, &p[4], 2, gu_map, 2 * c.intermediate, true, &gu);
  }
  if (rc == ALM_OK) {
    part = "down";
    rc = build_qweight(m->ctx, &p[6], 1, identity_map(c.hidden), c.hidden, true, &dn);
  }
  // row-layout copies for the batched prefill (dense tcgen05 path)
  DenseLayer D;
  if (rc == ALM_OK && dense_prefill_ok(m, p)) {
    const int I = c.intermediate;
    auto qkv_rows = [qd, kd](int layout) {
      std::vector<int> mp(padded_rows(qd + 2 * kd, layout), -1);
      for (int r = 0; r < qd; ++r) mp[r] = r;
      for (int r = 0; r < kd; ++r) mp[qd + r] = (1 << 24) | r;
      for (int r = 0; r < kd; ++r) mp[qd + kd + r] = (2 << 24) | r;
      return mp;
    };
    auto gu_rows = [I](int layout) {
      std::vector<int> mp(padded_rows(2 * I, layout), -1);
      for (int j = 0; j < I; ++j) {
        mp[j] = j;
        mp[I + j] = (1 << 24) | j;
      }
      return mp;
    };
    part = "qkv (row layout)";
    rc = build_qweight(m->ctx, &p[0], 3, qkv_rows, qd + 2 * kd, true, &D.qkv, true);
    if (rc == ALM_OK) {
      part = "o (row layout)";
      rc = build_qweight(m->ctx, &p[3], 1, identity_map(c.hidden), c.hidden, true, &D.o, true);
    }
    if (rc == ALM_OK) {
      part = "gate/up (row layout)";
      rc = build_qweight(m->ctx, &p[4], 2, gu_rows, 2 * I, true, &D.gu, true);
    }
    if (rc == ALM_OK) {
      part = "down (row layout)";
      rc = build_qweight(m->ctx, &p[6], 1, identity_map(c.hidden), c.hidden, true, &D.down, true);
    }
  }
  if (rc != ALM_OK) g_err = "layer " + std::to_string(li) + " " + part + ": " + g_err;
  half *nin = nullptr, *npost = nullptr;
  if (rc == ALM_OK) rc = dev_alloc_t(&nin, c.hidden);
  if (rc == ALM_OK) rc = dev_alloc_t(&npost, c.hidden);
  if (rc == ALM_OK && (cudaMemcpy(nin, n_in_host, c.hidden * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
                       cudaMemcpy(npost, n_post_host, c.hidden * 2, cudaMemcpyHostToDevice) != cudaSuccess))
    rc = fail(ALM_ERR_CUDA, "norm upload failed");
  if (rc != ALM_OK) {
    alm_qweight_free(qkv);
    alm_qweight_free(o);
    alm_qweight_free(gu);
    alm_qweight_free(dn);
    free_dense(D);
    dev_free(nin);
    dev_free(npost);
    return rc;
  }
  free_dense(m->dense[li]);
  m->dense[li] = D;
  alm_qweight_free(L.qkv);
  alm_qweight_free(L.o);
  alm_qweight_free(L.gu);
  alm_qweight_free(L.down);
  dev_free(L.n_in);
  dev_free(L.n_post);
  L = Layer{qkv, o, gu, dn, nin, npost};
  m->finalized = false;
  return ALM_OK;
}

int alm_model_set_embed(alm_model* m, const void* table_host, const void* scale_host, int bits, int block) {
  ALM_REQ(m && table_host, "null argument");
  const alm_model_config& c = m->cfg;
  ALM_REQ(bits == 16 || ((bits == 4 || bits == 8) && scale_host && block > 0 && c.hidden % block == 0),
          "embedding must be fp16 or int4/int8 with a block dividing hidden");
  DeviceGuard g(m->ctx->device);
  dev_free(m->embed_table);
  dev_free(m->embed_scale);
  m->embed_table = nullptr;
  m->embed_scale = nullptr;
  const int row_bytes = bits == 16 ? c.hidden * 2 : bits == 8 ? c.hidden : c.hidden / 2;
  const size_t nb = static_cast<size_t>(c.vocab) * row_bytes;
  ALM_TRY(dev_alloc(&m->embed_table, nb));
  ALM_CUDA(cudaMemcpy(m->embed_table, table_host, nb, cudaMemcpyHostToDevice));
  m->embed_bits = bits;
  m->embed_block = bits == 16 ? c.hidden : block;
  m->embed_nsb = bits == 16 ? 0 : c.hidden / block;
  m->embed_row_bytes = row_bytes;
  if (bits != 16) {
    const size_t sb = static_cast<size_t>(c.vocab) * m->embed_nsb * sizeof(half);
    ALM_TRY(dev_alloc(reinterpret_cast<void**>(&m->embed_scale), sb));
    ALM_CUDA(cudaMemcpy(m->embed_scale, scale_host, sb, cudaMemcpyHostToDevice));
  }
  m->finalized = false;
  return ALM_OK;
}

int alm_model_set_final_norm(alm_model* m, const uint16_t* w_host) {
  ALM_REQ(m && w_host, "null argument");
  DeviceGuard g(m->ctx->device);
  dev_free(m->final_norm);
  m->final_norm = nullptr;
  ALM_TRY(dev_alloc_t(&m->final_norm, m->cfg.hidden));
  ALM_CUDA(cudaMemcpy(m->final_norm, w_host, m->cfg.hidden * 2, cudaMemcpyHostToDevice));
  return ALM_OK;
}

int alm_model_set_head(alm_model* m, const alm_proj_src* head) {
  ALM_REQ(m && head, "null argument");
  ALM_REQ(head->out == (m->tp ? m->vocab_local : m->cfg.vocab) && head->in_real == m->cfg.hidden,
          "head must be (vocab, hidden), or (vocab_local, hidden) for a tensor-parallel shard");
  DeviceGuard g(m->ctx->device);
  alm_qweight* w = nullptr;
  ALM_TRY(build_qweight(m->ctx, head, 1, identity_map(head->out), head->out, true, &w));
  alm_qweight_free(m->head);
  m->head = w;
  m->finalized = false;
  return ALM_OK;
}

int alm_model_set_tp(alm_model* m, int vocab_offset, int vocab_local) {
  ALM_REQ(m, "null model");
  ALM_REQ(m->ctx->tp_comm, "tensor parallelism not initialised on the context (alm_ctx_init_tp)");
  ALM_REQ(vocab_local >= 1 && vocab_offset >= 0 && vocab_offset + vocab_local <= m->cfg.vocab,
          "vocabulary slice out of range");
  ALM_REQ(vocab_local * m->ctx->tp_world == m->cfg.vocab,
          "the vocabulary must split evenly over the ranks (vocab_local * world == vocab)");
  ALM_REQ(!m->head, "alm_model_set_tp comes before alm_model_set_head");
  m->tp = true;
  m->vocab_offset = vocab_offset;
  m->vocab_local = vocab_local;
  m->finalized = false;
  return ALM_OK;
}

int alm_model_finalize(alm_model* m) {
  ALM_REQ(m, "null model");
  DeviceGuard g(m->ctx->device);
  const alm_model_config& c = m->cfg;
  if (!m->embed_table) return fail(ALM_ERR_STATE, "embedding not set");
  if (!m->final_norm) return fail(ALM_ERR_STATE, "final norm not set");
  if (m->tp && !m->head)
    return fail(ALM_ERR_STATE, "a tensor-parallel shard needs its head rows (alm_model_set_head)");
  if (!m->head) {
    // tied head: the embedding table in the tile layout
    alm_proj_src s{m->embed_table, m->embed_scale, m->embed_bits, m->embed_block, c.vocab, c.hidden, c.hidden};
    // the sources must be host memory: copy the device table back once
    const size_t nb = static_cast<size_t>(c.vocab) * m->embed_row_bytes;
    std::vector<uint8_t> host_tbl(nb);
    ALM_CUDA(cudaMemcpy(host_tbl.data(), m->embed_table, nb, cudaMemcpyDeviceToHost));
    std::vector<uint8_t> host_scl;
    if (m->embed_bits != 16) {
      host_scl.resize(static_cast<size_t>(c.vocab) * m->embed_nsb * sizeof(half));
      ALM_CUDA(cudaMemcpy(host_scl.data(), m->embed_scale, host_scl.size(), cudaMemcpyDeviceToHost));
    }
    s.packed_host = host_tbl.data();
    s.scale_host = m->embed_bits != 16 ? host_scl.data() : nullptr;
    alm_qweight* w = nullptr;
    ALM_TRY(build_qweight(m->ctx, &s, 1, identity_map(c.vocab), c.vocab, true, &w));
    m->head = w;
  }
  Work& ws = m->ws;
  if (!ws.x0) {
    const int H = c.hidden, ht = n_h_tiles(m), qd = c.heads * c.head_dim;
    // row buffers hold the largest multi-sequence pass
    const size_t R = kMaxPassRows;
    ALM_TRY(dev_alloc_t(&ws.tokens, R));
    ALM_TRY(dev_alloc_t(&ws.rows, R));
    ALM_TRY(dev_alloc_t(&ws.seqs, kMaxRows));
    ALM_TRY(dev_alloc_t(&ws.u_rows, R));
    ALM_CUDA(cudaMallocHost(&ws.seq_host, kSeqStaging));
    ALM_TRY(dev_alloc_t(&ws.pos, 1));
    ALM_TRY(dev_alloc_t(&ws.err, 1));
    ALM_CUDA(cudaMemset(ws.err, 0, sizeof(int)));
    ALM_TRY(dev_alloc_t(&ws.x0, R * H));
    ALM_TRY(dev_alloc_t(&ws.s1, R * H));
    ALM_TRY(dev_alloc_t(&ws.s2, R * H));
    ALM_TRY(dev_alloc_t(&ws.ss1, R * ht));
    ALM_TRY(dev_alloc_t(&ws.ss2, R * ht));
    ALM_TRY(dev_alloc_t(&ws.q, R * qd));
    ALM_TRY(dev_alloc_t(&ws.ctx, R * qd));
    ALM_TRY(dev_alloc_t(&ws.h, R * c.intermediate));
    ALM_TRY(dev_alloc_t(&ws.xn, R * H));
    ALM_TRY(dev_alloc_t(&ws.xout, R * H));
    ALM_TRY(dev_alloc_t(&ws.logits, R * c.vocab));
    ALM_TRY(dev_alloc_t(&ws.argmax, R));
    ALM_CUDA(cudaMallocHost(reinterpret_cast<void**>(&ws.pinned), 64 * sizeof(int)));
  }
  if (m->tp && !ws.o32) {
    const int world = m->ctx->tp_world;
    ALM_TRY(dev_alloc_t(&ws.o32, static_cast<size_t>(kMaxRows) * c.hidden));
    ALM_TRY(dev_alloc_t(&ws.tp_pairs, static_cast<size_t>(2 * kMaxRows) * (world + 1)));
    ALM_TRY(dev_alloc_t(&ws.logits_local, static_cast<size_t>(kMaxRows) * m->vocab_local));
    ALM_TRY(dev_alloc_t(&ws.logits_gather, static_cast<size_t>(kMaxRows) * m->vocab_local * world));
  }
  // per-CTA argmax partials of the head
  const int n_am = gemv_out_blocks(m->head->t);
  if (n_am > ws.n_am) {
    dev_free(ws.am_val);
    dev_free(ws.am_idx);
    ws.am_val = nullptr;
    ws.am_idx = nullptr;
    ALM_TRY(dev_alloc_t(&ws.am_val, static_cast<size_t>(kMaxPassRows) * n_am));
    ALM_TRY(dev_alloc_t(&ws.am_idx, static_cast<size_t>(kMaxPassRows) * n_am));
  }
  ws.n_am = n_am;
  size_t need = split_need(m->head);
  for (const Layer& L : m->layers)
    need = std::max({need, split_need(L.qkv), split_need(L.o), split_need(L.gu), split_need(L.down)});
  ALM_TRY(ensure_part(ws, need));
  ALM_TRY(build_forward(m));
  ALM_TRY(build_cluster_fwd(m));
  if (m->tp) {   // the single-launch forwards have no collectives
    m->fwd_grid = 0;
    m->cf_ok = false;
  }
  m->finalized = true;
  return ALM_OK;
}

// ---- KV ------------------------------------------------------------------------
int alm_kv_create(alm_ctx* ctx, const alm_model* m, int max_len, int page_size, alm_kv** out) {
  return alm_kv_create_slots(ctx, m, 1, max_len, page_size, out);
}

int alm_kv_create_slots(alm_ctx* ctx, const alm_model* m, int n_slots, int max_len, int page_size, alm_kv** out) {
  ALM_REQ(ctx && m && out, "null argument");
  ALM_REQ(max_len > 0 && page_size > 0 && page_size <= 256, "invalid kv geometry");
  ALM_REQ(n_slots >= 1 && n_slots <= 4096, "n_slots must be in 1..4096");
  DeviceGuard g(ctx->device);
  auto* kv = new alm_kv();
  kv->ctx = ctx;
  kv->n_layers = m->cfg.layers;
  kv->kv_heads = m->cfg.kv_heads;
  kv->head_dim = m->cfg.head_dim;
  kv->page_size = page_size;
  kv->n_slots = n_slots;
  kv->pages_per_slot = (max_len + page_size - 1) / page_size;
  kv->n_pages = n_slots * kv->pages_per_slot;
  kv->max_len = max_len;
  kv->layer_elems = static_cast<size_t>(kv->n_pages) * page_size * kv->kv_heads * kv->head_dim;
  int rc = dev_alloc_t(&kv->k, kv->layer_elems * kv->n_layers);
  if (rc == ALM_OK) rc = dev_alloc_t(&kv->v, kv->layer_elems * kv->n_layers);
  if (rc == ALM_OK) rc = dev_alloc_t(&kv->page_table, kv->n_pages);
  if (rc == ALM_OK) {
    std::vector<int> pt(kv->n_pages);
    for (int i = 0; i < kv->n_pages; ++i) pt[i] = i;
    if (cudaMemcpy(kv->page_table, pt.data(), pt.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
      rc = fail(ALM_ERR_CUDA, "page table upload failed");
  }
  if (rc == ALM_OK) rc = alm_kv_zero(kv);
  if (rc != ALM_OK) {
    alm_kv_destroy(kv);
    return rc;
  }
  *out = kv;
  return ALM_OK;
}

int alm_kv_destroy(alm_kv* kv) {
  if (!kv) return ALM_OK;
  DeviceGuard g(kv->ctx->device);
  cudaStreamSynchronize(kv->ctx->stream);
  dev_free(kv->k);
  dev_free(kv->v);
  dev_free(kv->page_table);
  delete kv;
  return ALM_OK;
}

int alm_kv_zero(alm_kv* kv) {
  ALM_REQ(kv, "null kv");
  DeviceGuard g(kv->ctx->device);
  ALM_CUDA(cudaMemsetAsync(kv->k, 0, kv->layer_elems * kv->n_layers * sizeof(half), kv->ctx->stream));
  ALM_CUDA(cudaMemsetAsync(kv->v, 0, kv->layer_elems * kv->n_layers * sizeof(half), kv->ctx->stream));
  ALM_CUDA(cudaStreamSynchronize(kv->ctx->stream));
  return ALM_OK;
}

static int kv_copy(alm_kv* kv, int slot, int layer, int pos0, int n, uint16_t* k_host, uint16_t* v_host,
                   const uint16_t* k_in, const uint16_t* v_in) {
  ALM_REQ(kv, "null kv");
  ALM_REQ(slot >= 0 && slot < kv->n_slots, "slot out of range");
  ALM_REQ(layer >= 0 && layer < kv->n_layers && pos0 >= 0 && n >= 0 && pos0 + n <= kv->max_len,
          "kv range out of bounds");
  DeviceGuard g(kv->ctx->device);
  const size_t row = static_cast<size_t>(kv->head_dim) * sizeof(half);
  std::vector<int> pt(kv->n_pages);
  ALM_CUDA(cudaMemcpy(pt.data(), kv->page_table, pt.size() * sizeof(int), cudaMemcpyDeviceToHost));
  for (int which = 0; which < 2; ++which) {
    half* base = (which == 0 ? kv->k : kv->v) + static_cast<size_t>(layer) * kv->layer_elems;
    uint16_t* out = which == 0 ? k_host : v_host;
    const uint16_t* in = which == 0 ? k_in : v_in;
    if (!out && !in) continue;
    for (int i = 0; i < n; ++i) {
      const int p = pos0 + i;
      for (int h = 0; h < kv->kv_heads; ++h) {
        const int page = pt[static_cast<size_t>(slot) * kv->pages_per_slot + p / kv->page_size];
        half* src = base + ((static_cast<size_t>(page) * kv->kv_heads + h) * kv->page_size +
                            p % kv->page_size) * kv->head_dim;
        const size_t off = (static_cast<size_t>(i) * kv->kv_heads + h) * kv->head_dim;
        if (out) ALM_CUDA(cudaMemcpy(out + off, src, row, cudaMemcpyDeviceToHost));
        else ALM_CUDA(cudaMemcpy(src, in + off, row, cudaMemcpyHostToDevice));
      }
    }
  }
  return ALM_OK;
}

int alm_kv_read(alm_kv* kv, int layer, int pos0, int n, uint16_t* k_host, uint16_t* v_host) {
  return kv_copy(kv, 0, layer, pos0, n, k_host, v_host, nullptr, nullptr);
}
int alm_kv_write(alm_kv* kv, int layer, int pos0, int n, const uint16_t* k_host, const uint16_t* v_host) {
  return kv_copy(kv, 0, layer, pos0, n, nullptr, nullptr, k_host, v_host);
}
int alm_kv_read_slot(alm_kv* kv, int slot, int layer, int pos0, int n, uint16_t* k_host, uint16_t* v_host) {
  return kv_copy(kv, slot, layer, pos0, n, k_host, v_host, nullptr, nullptr);
}

int alm_kv_set_pages(alm_kv* kv, int slot, const int32_t* pages_host, int n) {
  ALM_REQ(kv && pages_host, "null argument");
  ALM_REQ(slot >= 0 && slot < kv->n_slots, "slot out of range");
  ALM_REQ(n >= 1 && n <= kv->pages_per_slot, "page count out of range");
  for (int i = 0; i < n; ++i)
    ALM_REQ(pages_host[i] >= 0 && pages_host[i] < kv->n_pages, "page number out of range");
  DeviceGuard g(kv->ctx->device);
  ALM_CUDA(cudaStreamSynchronize(kv->ctx->stream));
  ALM_CUDA(cudaMemcpy(kv->page_table + static_cast<size_t>(slot) * kv->pages_per_slot, pages_host, n * sizeof(int),
                      cudaMemcpyHostToDevice));
  return ALM_OK;
}

// ---- forward --------------------------------------------------------------------
int alm_layer_forward(alm_model* m, int layer, alm_kv* kv, const uint16_t* x_host, int rows, int pos0,
                      uint16_t* out_host) {
  ALM_TRY(check_ready(m));
  ALM_REQ(x_host && out_host, "null argument");
  ALM_REQ(layer >= 0 && layer < m->cfg.layers, "layer index out of range");
  if (!m->layers[layer].qkv) return fail(ALM_ERR_STATE, "layer " + std::to_string(layer) + " not set");
  DeviceGuard g(m->ctx->device);
  ALM_TRY(check_kv(m, kv, rows, pos0));
  cudaStream_t st = m->ctx->stream;
  const size_t nb = static_cast<size_t>(rows) * m->cfg.hidden * sizeof(half);
  ALM_TRY(set_pos(m, pos0));
  ALM_CUDA(cudaMemcpyAsync(m->ws.x0, x_host, nb, cudaMemcpyHostToDevice, st));
  const bool pdl = m->ctx->pdl;
  ALM_TRY(enqueue_layer(m, layer, kv, rows, raw_in(m->ws.x0, m->cfg.hidden, m->cfg.hidden), pdl));
  const ActIn o = deferred_in(m, m->ws.s2, m->ws.ss2, m->layers[layer].n_post);
  ALM_CUDA(launch_rownorm(o, rows, nullptr, 0.f, m->ws.xout, m->cfg.hidden, pdl, st));
  ALM_CUDA(cudaMemcpyAsync(out_host, m->ws.xout, nb, cudaMemcpyDeviceToHost, st));
  return sync_and_check(m);
}

int alm_head_logits(alm_model* m, const uint16_t* x_host, int rows, float* logits_host, int32_t* argmax_host) {
  ALM_TRY(check_ready(m));
  ALM_REQ(x_host, "null argument");
  ALM_REQ(rows >= 1 && rows <= kMaxRows, "rows must be in 1..16");
  DeviceGuard g(m->ctx->device);
  cudaStream_t st = m->ctx->stream;
  ALM_CUDA(cudaMemcpyAsync(m->ws.x0, x_host, static_cast<size_t>(rows) * m->cfg.hidden * 2,
                           cudaMemcpyHostToDevice, st));
  ALM_CUDA(launch_rownorm(raw_in(m->ws.x0, m->cfg.hidden, m->cfg.hidden), rows, m->final_norm, m->cfg.rms_eps,
                          m->ws.xn, m->cfg.hidden, m->ctx->pdl, st));
  m->tp_need_logits = logits_host != nullptr;
  const int rc = enqueue_head(m, rows, m->ctx->pdl);
  m->tp_need_logits = false;
  ALM_TRY(rc);
  ALM_TRY(sync_and_check(m));
  return copy_logits_out(m, rows, logits_host, argmax_host);
}

int alm_forward_trace(alm_model* m, alm_kv* kv, const int32_t* tokens_host, int rows, int pos0,
                      uint64_t* trace_host, int cap, int* n_barriers, int* n_ctas) {
  ALM_TRY(check_ready(m));
  ALM_REQ(tokens_host && trace_host && n_barriers && n_ctas, "null argument");
  ALM_TRY(check_layers(m));
  ALM_REQ(rows >= 1 && rows <= 8, "rows must be in 1..8");
  DeviceGuard g(m->ctx->device);
  if (rows == 1 && m->cf_ok && m->ctx->cluster) {
    // cluster forward: trace_host[0] = n, then n entries (label << 48 |
    // global ns) of CTA 0's decoding threads; from cap / 2 the same for its
    // weight producer
    ALM_TRY(check_kv(m, kv, rows, pos0));
    ALM_REQ(cap >= 64, "trace buffer too small");
    unsigned long long* dtrace = nullptr;
    ALM_TRY(dev_alloc_t(&dtrace, static_cast<size_t>(cap)));
    cudaStream_t st = m->ctx->stream;
    int rc = set_pos(m, pos0);
    if (rc == ALM_OK && cudaMemsetAsync(dtrace, 0, static_cast<size_t>(cap) * 8, st) != cudaSuccess)
      rc = fail(ALM_ERR_CUDA, "trace clear failed");
    if (rc == ALM_OK && cudaMemcpyAsync(m->ws.tokens, tokens_host, sizeof(int), cudaMemcpyHostToDevice, st) !=
                            cudaSuccess)
      rc = fail(ALM_ERR_CUDA, "token upload failed");
    FwdParams p = forward_params(m, kv, 1, false);
    p.trace = dtrace;
    p.trace_cap = cap;
    if (rc == ALM_OK && launch_cluster_fwd(p, m->cf_smem, false, st) != cudaSuccess)
      rc = fail(ALM_ERR_CUDA, "cluster forward launch failed");
    if (rc == ALM_OK) rc = sync_and_check(m);
    if (rc == ALM_OK && cudaMemcpy(trace_host, dtrace, static_cast<size_t>(cap) * 8, cudaMemcpyDeviceToHost) !=
                            cudaSuccess)
      rc = fail(ALM_ERR_CUDA, "trace download failed");
    dev_free(dtrace);
    if (rc != ALM_OK) return rc;
    *n_barriers = cap;
    *n_ctas = 1;
    return ALM_OK;
  }
  if (m->fwd_grid <= 0) return fail(ALM_ERR_STATE, "persistent forward kernel unavailable for this model");
  ALM_TRY(check_kv(m, kv, rows, pos0));
  const int nb = forward_barriers(m->cfg.layers, true);
  const size_t n = static_cast<size_t>(nb) * (m->fwd_grid + 1);
  ALM_REQ(cap >= 0 && static_cast<size_t>(cap) >= n, "trace buffer too small");
  unsigned long long* dtrace = nullptr;
  ALM_TRY(dev_alloc_t(&dtrace, n));
  cudaStream_t st = m->ctx->stream;
  int rc = set_pos(m, pos0);
  if (rc == ALM_OK && cudaMemcpyAsync(m->ws.tokens, tokens_host, rows * sizeof(int), cudaMemcpyHostToDevice, st) !=
                          cudaSuccess)
    rc = fail(ALM_ERR_CUDA, "token upload failed");
  if (rc == ALM_OK) rc = enqueue_forward_persistent(m, kv, rows, true, dtrace);
  if (rc == ALM_OK) rc = sync_and_check(m);
  if (rc == ALM_OK && cudaMemcpy(trace_host, dtrace, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost) !=
                          cudaSuccess)
    rc = fail(ALM_ERR_CUDA, "trace download failed");
  dev_free(dtrace);
  if (rc != ALM_OK) return rc;
  *n_barriers = nb;
  *n_ctas = m->fwd_grid;
  return ALM_OK;
}

int alm_sample(alm_ctx* ctx, const uint16_t* logits_host, int rows, int vocab, float temperature, float top_p,
               float min_p, const double* uniforms_host, int32_t* out_host) {
  ALM_REQ(ctx && logits_host && out_host && (uniforms_host || !(temperature > 0.f)), "null argument");
  ALM_REQ(rows >= 1 && vocab >= 1, "empty logits");
  ALM_REQ(top_p > 0.f && top_p <= 1.f, "top_p must be in (0, 1]");
  ALM_REQ(min_p >= 0.f && min_p < 1.f, "min_p must be in [0, 1)");
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  const size_t n = static_cast<size_t>(rows) * vocab;
  half* dl = nullptr;
  float* scr = nullptr;
  double* du = nullptr;
  int* dout = nullptr;
  int rc = dev_alloc_t(&dl, n);
  if (rc == ALM_OK) rc = dev_alloc_t(&scr, n);
  if (rc == ALM_OK) rc = dev_alloc_t(&du, static_cast<size_t>(rows));
  if (rc == ALM_OK) rc = dev_alloc_t(&dout, static_cast<size_t>(rows));
  if (rc == ALM_OK && (cudaMemcpyAsync(dl, logits_host, n * sizeof(half), cudaMemcpyHostToDevice, st) != cudaSuccess ||
                       (uniforms_host && cudaMemcpyAsync(du, uniforms_host, rows * sizeof(double),
                                                         cudaMemcpyHostToDevice, st) != cudaSuccess)))
    rc = fail(ALM_ERR_CUDA, "upload failed");
  if (rc == ALM_OK) {
    SampleArgs a;
    a.logits = dl;
    a.ld = vocab;
    a.vocab = vocab;
    a.temperature = temperature > 0.f ? std::max(temperature, 1e-9f) : 0.f;
    a.top_p = top_p;
    a.min_p = min_p;
    a.uniforms = du;
    a.scratch = scr;
    a.out = dout;
    const cudaError_t e = launch_sample(a, rows, false, st);
    if (e != cudaSuccess) rc = fail(ALM_ERR_CUDA, std::string("sample: ") + cudaGetErrorString(e));
  }
  if (rc == ALM_OK && (cudaMemcpyAsync(out_host, dout, rows * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                       cudaStreamSynchronize(st) != cudaSuccess))
    rc = fail(ALM_ERR_CUDA, "sample failed");
  dev_free(dl);
  dev_free(scr);
  dev_free(du);
  dev_free(dout);
  return rc;
}

int alm_probs(alm_ctx* ctx, const uint16_t* logits_host, int rows, int vocab, float temperature, float min_p,
              float* probs_host) {
  ALM_REQ(ctx && logits_host && probs_host, "null argument");
  ALM_REQ(rows >= 1 && vocab >= 1 && vocab <= kAccMaxChunks * 256, "rows >= 1 and 1 <= vocab <= 1048576");
  ALM_REQ(temperature > 0.f, "temperature must be positive");
  ALM_REQ(min_p >= 0.f && min_p < 1.f, "min_p must be in [0, 1)");
  DeviceGuard g(ctx->device);
  const size_t n = static_cast<size_t>(rows) * vocab;
  DevBufs b;
  half* lg = nullptr;
  float* pr = nullptr;
  ALM_TRY(b.get(&lg, n));
  ALM_TRY(b.get(&pr, n));
  ALM_CUDA(cudaMemcpyAsync(lg, logits_host, n * sizeof(half), cudaMemcpyHostToDevice, ctx->stream));
  ProbsArgs a;
  a.logits = lg;
  a.ld = vocab;
  a.probs = pr;
  a.ldp = vocab;
  a.vocab = vocab;
  a.t = std::max(temperature, 1e-9f);
  a.min_p = min_p;
  ALM_CUDA(launch_probs(a, rows, ctx->stream));
  ALM_CUDA(cudaMemcpyAsync(probs_host, pr, n * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
  ALM_CUDA(cudaStreamSynchronize(ctx->stream));
  return ALM_OK;
}

int alm_accept(alm_ctx* ctx, const uint16_t* target_logits_host, const float* draft_probs_host,
               const int32_t* draft_tokens_host, int k, int vocab, float temperature, float min_p,
               const double* uniforms_host, int32_t* out_tokens_host, int32_t* n_accepted_host) {
  ALM_REQ(ctx && target_logits_host && draft_probs_host && draft_tokens_host && uniforms_host && out_tokens_host &&
              n_accepted_host,
          "null argument");
  ALM_REQ(k >= 1 && k <= 31, "k must be in 1..31");
  ALM_REQ(vocab >= 1 && vocab <= kAccMaxChunks * 256, "vocab must be in 1..1048576");
  ALM_REQ(temperature > 0.f, "temperature must be positive");
  ALM_REQ(min_p >= 0.f && min_p < 1.f, "min_p must be in [0, 1)");
  for (int i = 0; i < k; ++i) ALM_REQ(draft_tokens_host[i] >= 0 && draft_tokens_host[i] < vocab, "draft token out of range");
  DeviceGuard g(ctx->device);
  cudaStream_t st = ctx->stream;
  const size_t vp = static_cast<size_t>(k + 1) * vocab, vq = static_cast<size_t>(k) * vocab;
  DevBufs b;
  half* lg = nullptr;
  float *p = nullptr, *q = nullptr;
  int *cand = nullptr, *tok = nullptr;
  double* u = nullptr;
  ALM_TRY(b.get(&lg, vp));
  ALM_TRY(b.get(&p, vp));
  ALM_TRY(b.get(&q, vq));
  ALM_TRY(b.get(&cand, static_cast<size_t>(k)));
  ALM_TRY(b.get(&tok, static_cast<size_t>(k + 2)));
  ALM_TRY(b.get(&u, static_cast<size_t>(k + 1)));
  ALM_CUDA(cudaMemcpyAsync(lg, target_logits_host, vp * sizeof(half), cudaMemcpyHostToDevice, st));
  ALM_CUDA(cudaMemcpyAsync(q, draft_probs_host, vq * sizeof(float), cudaMemcpyHostToDevice, st));
  ALM_CUDA(cudaMemcpyAsync(cand, draft_tokens_host, k * sizeof(int), cudaMemcpyHostToDevice, st));
  ALM_CUDA(cudaMemcpyAsync(u, uniforms_host, (k + 1) * sizeof(double), cudaMemcpyHostToDevice, st));
  ProbsArgs pa;
  pa.logits = lg;
  pa.ld = vocab;
  pa.probs = p;
  pa.ldp = vocab;
  pa.vocab = vocab;
  pa.t = std::max(temperature, 1e-9f);
  pa.min_p = min_p;
  ALM_CUDA(launch_probs(pa, k + 1, st));
  AcceptArgs aa;
  aa.p = p;
  aa.ldp = vocab;
  aa.q = q;
  aa.ldq = vocab;
  aa.cand = cand;
  aa.k = k;
  aa.vocab = vocab;
  aa.u = u;
  aa.tokens = tok;
  aa.n_acc = tok + k + 1;
  ALM_CUDA(launch_accept(aa, st));
  int host[33];
  ALM_CUDA(cudaMemcpyAsync(host, tok, (k + 2) * sizeof(int), cudaMemcpyDeviceToHost, st));
  ALM_CUDA(cudaStreamSynchronize(st));
  const int n = host[k + 1];
  for (int i = 0; i <= n; ++i) out_tokens_host[i] = host[i];
  *n_accepted_host = n;
  return ALM_OK;
}

int alm_model_sample(alm_model* m, int rows, float temperature, float top_p, float min_p,
                     const double* uniforms_host, int32_t* out_host) {
  return alm_model_sample_rows(m, 0, rows, temperature, top_p, min_p, uniforms_host, out_host);
}

int alm_model_sample_rows(alm_model* m, int row0, int rows, float temperature, float top_p, float min_p,
                          const double* uniforms_host, int32_t* out_host) {
  ALM_TRY(check_ready(m));
  ALM_REQ(out_host && (uniforms_host || !(temperature > 0.f)), "null argument");
  ALM_REQ(row0 >= 0 && rows >= 1 && row0 + rows <= kMaxPassRows, "rows must lie in 0..63");
  ALM_REQ(top_p > 0.f && top_p <= 1.f, "top_p must be in (0, 1]");
  ALM_REQ(min_p >= 0.f && min_p < 1.f, "min_p must be in [0, 1)");
  DeviceGuard g(m->ctx->device);
  ALM_TRY(ensure_sample_scratch(m));
  cudaStream_t st = m->ctx->stream;
  double* du = m->ws.u_rows;
  int rc = ALM_OK;
  if (uniforms_host &&
      cudaMemcpyAsync(du, uniforms_host, rows * sizeof(double), cudaMemcpyHostToDevice, st) != cudaSuccess)
    rc = fail(ALM_ERR_CUDA, "upload failed");
  if (rc == ALM_OK) {
    const float t = temperature > 0.f ? std::max(temperature, 1e-9f) : 0.f;
    SampleArgs sa = sample_args(m, t, top_p, min_p, du, nullptr, 0);
    sa.logits += static_cast<size_t>(row0) * sa.ld;
    sa.out += row0;
    const cudaError_t e = launch_sample(sa, rows, false, st);
    if (e != cudaSuccess) rc = fail(ALM_ERR_CUDA, std::string("sample: ") + cudaGetErrorString(e));
  }
  if (rc == ALM_OK && (cudaMemcpyAsync(out_host, m->ws.argmax + row0, rows * sizeof(int), cudaMemcpyDeviceToHost,
                                       st) !=
                           cudaSuccess ||
                       cudaStreamSynchronize(st) != cudaSuccess))
    rc = fail(ALM_ERR_CUDA, "sample failed");
  return rc;
}

// Rows of one multi-sequence pass: row groups of the M <= 16 GEMV up to
// kMaxPassRows; the tcgen05 decode weights' fused epilogues take 16.
static int max_pass_rows(const alm_model* m) { return m->ctx->tc ? kMaxRows : kMaxPassRows; }

// Check and upload a multi-sequence pass's rows and sequences (ws.rows,
// ws.seqs) and mark the model's next enqueue as that pass; *M_out = rows.
static int stage_seqs(alm_model* m, alm_kv* kv, int n_seq, const int32_t* slots, const int32_t* n_tok,
                      const int32_t* pos0, const int32_t* tokens_host, int* M_out) {
  ALM_REQ(!m->tp, "multi-sequence passes run on whole models");
  ALM_REQ(n_seq >= 1 && n_seq <= kMaxRows, "n_seq must be in 1..16");
  ALM_REQ(kv->n_layers == m->cfg.layers && kv->kv_heads == m->cfg.kv_heads && kv->head_dim == m->cfg.head_dim,
          "kv cache shape mismatch");
  const int gq = m->cfg.heads / m->cfg.kv_heads;
  std::vector<int2> rows;
  std::vector<AttnSeq> seqs(n_seq);
  int g = 0, pg = 0;
  for (int s = 0; s < n_seq; ++s) {
    ALM_REQ(slots[s] >= 0 && slots[s] < kv->n_slots, "slot out of range");
    for (int t = 0; t < s; ++t) ALM_REQ(slots[t] != slots[s], "two sequences of one pass share a slot");
    ALM_REQ(n_tok[s] >= 1 && pos0[s] >= 0, "every sequence needs rows at non-negative positions");
    ALM_REQ(static_cast<long long>(pos0[s]) + n_tok[s] <= kv->max_len &&
                static_cast<long long>(pos0[s]) + n_tok[s] <= m->cfg.max_len,
            "pos out of kv cache or rope table range");
    ALM_REQ(static_cast<int>(rows.size()) + n_tok[s] <= max_pass_rows(m), "more rows than alm_model_max_pass_rows");
    const int off = slots[s] * kv->pages_per_slot;
    seqs[s] = AttnSeq{static_cast<int>(rows.size()), n_tok[s], pos0[s], off, g, pg};
    for (int t = 0; t < n_tok[s]; ++t) rows.push_back(make_int2(pos0[s] + t, off));
    g += (n_tok[s] * gq + kAttnRows - 1) / kAttnRows;
    pg += (n_tok[s] * gq + kPvRows - 1) / kPvRows;
  }
  ALM_TRY(ensure_attn(m, kv->max_len));
  // one pinned staging area, three async copies on the model's stream (the
  // previous call on this stream has finished: every call ends synchronised)
  const int M = static_cast<int>(rows.size());
  unsigned char* h = m->ws.seq_host;
  std::memcpy(h, rows.data(), M * sizeof(int2));
  std::memcpy(h + kMaxPassRows * sizeof(int2), seqs.data(), n_seq * sizeof(AttnSeq));
  std::memcpy(h + kMaxPassRows * (sizeof(int2) + sizeof(AttnSeq)), tokens_host, M * sizeof(int));
  cudaStream_t st = m->ctx->stream;
  ALM_CUDA(cudaMemcpyAsync(m->ws.rows, h, M * sizeof(int2), cudaMemcpyHostToDevice, st));
  ALM_CUDA(cudaMemcpyAsync(m->ws.seqs, h + kMaxPassRows * sizeof(int2), n_seq * sizeof(AttnSeq),
                           cudaMemcpyHostToDevice, st));
  ALM_CUDA(cudaMemcpyAsync(m->ws.tokens, h + kMaxPassRows * (sizeof(int2) + sizeof(AttnSeq)), M * sizeof(int),
                           cudaMemcpyHostToDevice, st));
  m->ms_n_seq = n_seq;
  m->ms_n_rg = g;
  m->ms_n_pg = pg;
  *M_out = static_cast<int>(rows.size());
  return ALM_OK;
}

static void clear_seqs(alm_model* m) { m->ms_n_seq = m->ms_n_rg = m->ms_n_pg = 0; }

// Several sequences in one pass: sequence s has n_tok[s] rows (its tokens
// in order in tokens_host) at positions pos0[s] .. of KV slot slots[s].  The
// weights stream once for all rows; every row's result equals its
// sequence's own forward (rows never mix in a reduction).
int alm_forward_seqs(alm_model* m, alm_kv* kv, int n_seq, const int32_t* slots, const int32_t* n_tok,
                     const int32_t* pos0, const int32_t* tokens_host, float* logits_host, int32_t* argmax_host) {
  ALM_TRY(check_ready(m));
  ALM_REQ(kv && slots && n_tok && pos0 && tokens_host, "null argument");
  ALM_TRY(check_layers(m));
  DeviceGuard gd(m->ctx->device);
  int M = 0;
  ALM_TRY(stage_seqs(m, kv, n_seq, slots, n_tok, pos0, tokens_host, &M));
  const bool head = logits_host != nullptr || argmax_host != nullptr;
  const alm_model::MsKey key{kv->k, kv->v, kv->page_table, kv->max_len, kv->pages_per_slot, M, n_seq, m->ms_n_rg,
                             m->ms_n_pg, head ? 1 : 0};
  cudaStream_t st = m->ctx->stream;
  int rc = ALM_OK;
  auto it = m->ms_graphs.find(key);
  if (it == m->ms_graphs.end()) {
    // first pass of this shape: capture it (the staging copies are already queued)
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      rc = fail(ALM_ERR_CUDA, "graph capture failed to start");
    } else {
      rc = enqueue_forward(m, kv, M, head, m->ctx->pdl);
      const cudaError_t e = cudaStreamEndCapture(st, &graph);
      if (rc == ALM_OK && e != cudaSuccess) rc = fail(ALM_ERR_CUDA, std::string("capture: ") + cudaGetErrorString(e));
      if (rc == ALM_OK && cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess)
        rc = fail(ALM_ERR_CUDA, "instantiate of a multi-sequence pass failed");
      if (graph) cudaGraphDestroy(graph);
    }
    if (rc == ALM_OK) it = m->ms_graphs.emplace(key, exec).first;
  }
  if (rc == ALM_OK && cudaGraphLaunch(it->second, st) != cudaSuccess) rc = fail(ALM_ERR_CUDA, "pass launch failed");
  clear_seqs(m);
  ALM_TRY(rc);
  ALM_TRY(sync_and_check(m));
  return copy_logits_out(m, M, logits_host, argmax_host);
}

// Fill the KV cache for positions pos0 .. pos0 + n - 1 from the tokens
// (androidllm/engine.py:345-361 runs them as n single-token forwards):
// chunks of up to 256 rows through the dense path when the model has its
// row-layout copies (a tail of at most 16 rows, or any chunk without them,
// through the M <= 16 forward).  No logits.
int alm_prefill(alm_model* m, alm_kv* kv, const int32_t* tokens_host, int n, int pos0) {
  return alm_prefill_slot(m, kv, 0, tokens_host, n, pos0);
}

int alm_prefill_slot(alm_model* m, alm_kv* kv, int slot, const int32_t* tokens_host, int n, int pos0) {
  ALM_TRY(check_ready(m));
  ALM_REQ(kv && slot >= 0 && slot < kv->n_slots, "slot out of range");
  ALM_REQ(tokens_host && kv, "null argument");
  ALM_TRY(check_layers(m));
  ALM_REQ(n >= 1, "n must be positive");
  ALM_REQ(kv->n_layers == m->cfg.layers && kv->kv_heads == m->cfg.kv_heads && kv->head_dim == m->cfg.head_dim,
          "kv cache shape mismatch");
  ALM_REQ(pos0 >= 0 && static_cast<long long>(pos0) + n <= kv->max_len, "pos out of kv cache range");
  ALM_REQ(static_cast<long long>(pos0) + n <= m->cfg.max_len, "pos out of rope table range");
  DeviceGuard g(m->ctx->device);
  ALM_TRY(ensure_attn(m, kv->max_len));
  const bool dense = dense_ready(m);
  if (dense) ALM_TRY(ensure_prefill(m, kv->max_len));
  cudaStream_t st = m->ctx->stream;
  for (int done = 0; done < n;) {
    const int rows = std::min(n - done, dense ? kMaxDenseRows : kMaxRows);
    const int p = pos0 + done;
    ALM_TRY(set_pos(m, p));
    if (rows > kMaxRows) {
      ALM_CUDA(cudaMemcpyAsync(m->pf.tokens, tokens_host + done, rows * sizeof(int), cudaMemcpyHostToDevice, st));
      ALM_TRY(enqueue_prefill_dense(m, kv, rows, p, slot));
    } else if (slot != 0) {
      // a short chunk of another slot: a one-sequence multi-sequence pass
      int M = 0;
      ALM_TRY(stage_seqs(m, kv, 1, &slot, &rows, &p, tokens_host + done, &M));
      const int rc = enqueue_forward(m, kv, rows, false, m->ctx->pdl);
      clear_seqs(m);
      ALM_TRY(rc);
    } else {
      ALM_CUDA(cudaMemcpyAsync(m->ws.tokens, tokens_host + done, rows * sizeof(int), cudaMemcpyHostToDevice, st));
      m->pv_one_span = p + rows <= kPvSplit;
      const int rc = enqueue_forward(m, kv, rows, false, m->ctx->pdl);
      m->pv_one_span = false;
      ALM_TRY(rc);
    }
    ALM_TRY(sync_and_check(m));
    done += rows;
  }
  return ALM_OK;
}

int alm_ctx_set_dense_prefill(alm_ctx* ctx, int enable) {
  ALM_REQ(ctx, "null context");
  ctx->dense_prefill = enable != 0;
  return ALM_OK;
}

int alm_model_max_pass_rows(const alm_model* m, int* rows) {
  ALM_REQ(m && rows, "null argument");
  *rows = m->tp ? 0 : max_pass_rows(m);
  return ALM_OK;
}

int alm_model_dense_prefill(const alm_model* m, int* dense) {
  ALM_REQ(m && dense, "null argument");
  *dense = dense_ready(m) ? 1 : 0;
  return ALM_OK;
}

int alm_forward(alm_model* m, alm_kv* kv, const int32_t* tokens_host, int rows, int pos0, float* logits_host,
                int32_t* argmax_host) {
  ALM_TRY(check_ready(m));
  ALM_REQ(tokens_host, "null argument");
  ALM_TRY(check_layers(m));
  DeviceGuard g(m->ctx->device);
  ALM_TRY(check_kv(m, kv, rows, pos0));
  cudaStream_t st = m->ctx->stream;
  ALM_TRY(set_pos(m, pos0));
  ALM_CUDA(cudaMemcpyAsync(m->ws.tokens, tokens_host, rows * sizeof(int), cudaMemcpyHostToDevice, st));
  const bool head = logits_host != nullptr || argmax_host != nullptr;
  m->tp_need_logits = logits_host != nullptr;
  m->pv_one_span = pos0 + rows <= kPvSplit;
  const int rc = enqueue_forward(m, kv, rows, head, m->ctx->pdl);
  m->tp_need_logits = false;
  m->pv_one_span = false;
  ALM_TRY(rc);
  ALM_TRY(sync_and_check(m));
  return copy_logits_out(m, rows, logits_host, argmax_host);
}

// ---- speculative decoding -----------------------------------------------------------
// The speculative step with min(1, p/q) rejection sampling: every draft
// candidate is an inverse-CDF draw from the draft's softmax row q_i (draw i),
// the verify rows' softmax rows p_0..p_k go to the acceptance kernel with
// draws k..2k (accept i, then the resample); the cursor advances 2k + 1.
static int enqueue_spec_step_rejection(alm_spec* s) {
  alm_model* d = s->draft;
  alm_model* t = s->target;
  cudaStream_t st = t->ctx->stream;
  const int V = t->cfg.vocab;
  float* p_rows = s->probs;
  float* q_rows = s->probs + static_cast<size_t>(s->k + 1) * V;
  const int r0 = s->refresh ? 2 : 1;   // rows of draft forward 0; its candidate is the last
  for (int i = 0; i < s->k; ++i) {
    const int rows = i == 0 ? r0 : 1;
    prof_role(0);
    ALM_CUDA(launch_spec_prep_draft(s->state, s->cand, d->ws.argmax, i, d->ws.tokens, d->ws.pos,
                                    i == 1 ? r0 - 1 : 0, s->refresh ? 1 : 0, st));
    prof_mark(ALM_OP_SPEC_PREP, 1);
    prof_role(1);
    ALM_TRY(enqueue_forward(d, s->dkv, rows, true, d->ctx->pdl));
    ProbsArgs pa;
    pa.logits = d->ws.logits + static_cast<size_t>(rows - 1) * V;
    pa.ld = V;
    pa.probs = q_rows + static_cast<size_t>(i) * V;
    pa.ldp = V;
    pa.vocab = V;
    pa.t = s->temperature;
    pa.min_p = s->min_p;
    ALM_CUDA(launch_probs(pa, 1, st));
    prof_mark(ALM_OP_SAMPLE, 1);
    DrawArgs da;
    da.probs = pa.probs;
    da.vocab = V;
    da.u = s->uniforms;
    da.cursor = s->state + 4;
    da.u_offset = i;
    da.out = d->ws.argmax + (rows - 1);
    ALM_CUDA(launch_draw(da, st));
    prof_mark(ALM_OP_SAMPLE, 1);
  }
  prof_role(0);
  ALM_CUDA(launch_spec_prep_verify(s->state, s->cand, d->ws.argmax, s->k, t->ws.tokens, t->ws.pos,
                                   s->k == 1 ? r0 - 1 : 0, st));
  prof_mark(ALM_OP_SPEC_PREP, s->k + 1);
  prof_role(2);
  ALM_TRY(enqueue_forward(t, s->tkv, s->k + 1, true, t->ctx->pdl));
  ProbsArgs pa;
  pa.logits = t->ws.logits;
  pa.ld = V;
  pa.probs = p_rows;
  pa.ldp = V;
  pa.vocab = V;
  pa.t = s->temperature;
  pa.min_p = s->min_p;
  ALM_CUDA(launch_probs(pa, s->k + 1, st));
  prof_mark(ALM_OP_SAMPLE, s->k + 1);
  prof_role(0);
  AcceptArgs aa;
  aa.p = p_rows;
  aa.ldp = V;
  aa.q = q_rows;
  aa.ldq = V;
  aa.cand = s->cand;
  aa.k = s->k;
  aa.vocab = V;
  aa.u = s->uniforms;
  aa.cursor = s->state + 4;
  aa.u_offset = s->k;
  aa.state = s->state;
  aa.ring = s->out_tokens;
  aa.ring_acc = s->out_acc;
  aa.cap_tokens = s->cap_tokens;
  aa.cap_steps = s->cap_steps;
  aa.cursor_advance = 2 * s->k + 1;
  ALM_CUDA(launch_accept(aa, st));
  prof_mark(ALM_OP_SPEC_ACCEPT, s->k + 1);
  return ALM_OK;
}

static int enqueue_spec_step(alm_spec* s) {
  if (s->rejection && s->temperature > 0.f) return enqueue_spec_step_rejection(s);
  alm_model* d = s->draft;
  alm_model* t = s->target;
  cudaStream_t st = t->ctx->stream;
  const bool sampled = s->temperature > 0.f;
  const int V = d->cfg.vocab;
  const int r0 = s->refresh ? 2 : 1;   // rows of draft forward 0; its candidate is the last
  for (int i = 0; i < s->k; ++i) {
    const int rows = i == 0 ? r0 : 1;
    prof_role(0);
    ALM_CUDA(launch_spec_prep_draft(s->state, s->cand, d->ws.argmax, i, d->ws.tokens, d->ws.pos,
                                    i == 1 ? r0 - 1 : 0, s->refresh ? 1 : 0, st));
    prof_mark(ALM_OP_SPEC_PREP, 1);
    prof_role(1);
    ALM_TRY(enqueue_forward(d, s->dkv, rows, true, d->ctx->pdl));
    // draft candidate i: the draft's sample of its last row, draw k-step offset i
    if (sampled) {
      SampleArgs sa = sample_args(d, s->temperature, s->top_p, s->min_p, s->uniforms, s->state + 4, i);
      sa.logits += static_cast<size_t>(rows - 1) * V;
      sa.out += rows - 1;
      ALM_CUDA(launch_sample(sa, 1, false, st));
      prof_mark(ALM_OP_SAMPLE, 1);
    }
  }
  prof_role(0);
  ALM_CUDA(launch_spec_prep_verify(s->state, s->cand, d->ws.argmax, s->k, t->ws.tokens, t->ws.pos,
                                   s->k == 1 ? r0 - 1 : 0, st));
  prof_mark(ALM_OP_SPEC_PREP, s->k + 1);
  prof_role(2);
  ALM_TRY(enqueue_forward(t, s->tkv, s->k + 1, true, t->ctx->pdl));
  // target row j: the target's sample with draw k + j
  if (sampled) {
    ALM_CUDA(launch_sample(sample_args(t, s->temperature, s->top_p, s->min_p, s->uniforms, s->state + 4, s->k),
                           s->k + 1, false, st));
    prof_mark(ALM_OP_SAMPLE, s->k + 1);
  }
  prof_role(0);
  ALM_CUDA(launch_spec_accept_greedy(s->state, s->cand, t->ws.argmax, s->k, s->out_tokens, s->out_acc,
                                     s->cap_tokens, s->cap_steps, sampled ? 1 : 0, st));
  prof_mark(ALM_OP_SPEC_ACCEPT, s->k + 1);
  return ALM_OK;
}

// Capture one step graph into *exec (destroyed first if set).
static int capture_step_graph(alm_spec* s, cudaGraphExec_t* exec, int* n_kernels) {
  if (*exec) {
    cudaGraphExecDestroy(*exec);
    *exec = nullptr;
  }
  cudaStream_t st = s->target->ctx->stream;
  cudaGraph_t graph = nullptr;
  if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
    return fail(ALM_ERR_CUDA, "graph capture failed to start");
  // the sampler reads the target's full logits rows
  s->target->tp_need_logits = s->temperature > 0.f;
  int rc = enqueue_spec_step(s);
  s->target->tp_need_logits = false;
  cudaError_t e = cudaStreamEndCapture(st, &graph);
  if (rc == ALM_OK && e != cudaSuccess) rc = fail(ALM_ERR_CUDA, std::string("capture: ") + cudaGetErrorString(e));
  if (rc == ALM_OK) {
    size_t n_nodes = 0;
    cudaGraphGetNodes(graph, nullptr, &n_nodes);
    std::vector<cudaGraphNode_t> nodes(n_nodes);
    if (n_nodes) cudaGraphGetNodes(graph, nodes.data(), &n_nodes);
    int n = 0;
    for (cudaGraphNode_t nd : nodes) {
      cudaGraphNodeType ty;
      if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++n;
    }
    if (n_kernels) *n_kernels = n;
    e = cudaGraphInstantiate(exec, graph, 0);
    if (e != cudaSuccess) rc = fail(ALM_ERR_CUDA, std::string("instantiate: ") + cudaGetErrorString(e));
  }
  if (graph) cudaGraphDestroy(graph);
  return rc;
}

// (Re)capture the step graphs for the decoder's current sampling settings:
// the general one and, when a KV cache is longer than one P.V span, the
// one-span variant.
static int capture_spec_graph(alm_spec* s) {
  if (s->temperature > 0.f) {
    ALM_TRY(ensure_sample_scratch(s->target));
    ALM_TRY(ensure_sample_scratch(s->draft));
  }
  if (s->rejection && !s->probs)
    ALM_TRY(dev_alloc_t(&s->probs, static_cast<size_t>(2 * s->k + 1) * s->target->cfg.vocab));
  s->n_kernels = 0;
  ALM_TRY(capture_step_graph(s, &s->graph, &s->n_kernels));
  if (s->graph_short) {
    cudaGraphExecDestroy(s->graph_short);
    s->graph_short = nullptr;
  }
  if (s->tkv->max_len > kPvSplit || s->dkv->max_len > kPvSplit) {
    s->target->pv_one_span = s->draft->pv_one_span = true;
    const int rc = capture_step_graph(s, &s->graph_short, nullptr);
    s->target->pv_one_span = s->draft->pv_one_span = false;
    ALM_TRY(rc);
  }
  return ALM_OK;
}

// The step graph for n_steps steps from position pos: the one-span variant
// when no pass of them reaches past one P.V span.
static cudaGraphExec_t step_graph(const alm_spec* s, int pos, int n_steps) {
  const long long last = static_cast<long long>(pos) + static_cast<long long>(n_steps) * (s->k + 1) + s->k + 1;
  return (s->graph_short && last <= kPvSplit) ? s->graph_short : s->graph;
}

int alm_spec_create(alm_model* target, alm_model* draft, alm_kv* target_kv, alm_kv* draft_kv, int k,
                    alm_spec** out) {
  ALM_TRY(check_ready(target));
  ALM_TRY(check_ready(draft));
  ALM_TRY(check_layers(target));
  ALM_TRY(check_layers(draft));
  ALM_REQ(out, "null argument");
  ALM_REQ(target->ctx == draft->ctx, "target and draft must share a context");
  ALM_REQ(k >= 1 && k + 1 <= kMaxRows, "k must be in 1..15");
  ALM_REQ(target->cfg.vocab == draft->cfg.vocab, "target and draft vocabularies differ");
  DeviceGuard g(target->ctx->device);
  ALM_TRY(check_kv(target, target_kv, k + 1, 0));
  ALM_TRY(check_kv(draft, draft_kv, 1, 0));
  auto* s = new alm_spec();
  s->target = target;
  s->draft = draft;
  s->tkv = target_kv;
  s->dkv = draft_kv;
  s->k = k;
  s->cap_steps = 1024;
  s->cap_tokens = s->cap_steps * (k + 1);
  int rc = dev_alloc_t(&s->state, 8);
  if (rc == ALM_OK) rc = dev_alloc_t(&s->cand, k);
  if (rc == ALM_OK) rc = dev_alloc_t(&s->out_tokens, s->cap_tokens);
  if (rc == ALM_OK) rc = dev_alloc_t(&s->out_acc, s->cap_steps);
  if (rc == ALM_OK && cudaMallocHost(reinterpret_cast<void**>(&s->pinned),
                                     (4 + s->cap_tokens + s->cap_steps) * sizeof(int)) != cudaSuccess)
    rc = fail(ALM_ERR_CUDA, "pinned allocation failed");
  if (rc == ALM_OK && cudaMemset(s->state, 0, 8 * sizeof(int)) != cudaSuccess)
    rc = fail(ALM_ERR_CUDA, "state init failed");
  if (rc == ALM_OK) rc = capture_spec_graph(s);
  if (rc != ALM_OK) {
    alm_spec_destroy(s);
    return rc;
  }
  *out = s;
  return ALM_OK;
}

int alm_spec_destroy(alm_spec* s) {
  if (!s) return ALM_OK;
  DeviceGuard g(s->target->ctx->device);
  cudaStreamSynchronize(s->target->ctx->stream);
  if (s->graph) cudaGraphExecDestroy(s->graph);
  if (s->graph_short) cudaGraphExecDestroy(s->graph_short);
  dev_free(s->state);
  dev_free(s->cand);
  dev_free(s->out_tokens);
  dev_free(s->out_acc);
  dev_free(s->uniforms);
  dev_free(s->probs);
  if (s->pinned) cudaFreeHost(s->pinned);
  delete s;
  return ALM_OK;
}

int alm_spec_begin_prev(alm_spec* s, int32_t prev_token, int32_t token, int pos) {
  ALM_REQ(s, "null spec");
  ALM_REQ(prev_token >= 0 && prev_token < s->target->cfg.vocab, "token out of range");
  ALM_REQ(pos >= 1, "the previous token needs pos >= 1");
  DeviceGuard g(s->target->ctx->device);
  s->pinned[4] = prev_token;
  ALM_CUDA(cudaMemcpyAsync(s->state + 5, s->pinned + 4, sizeof(int), cudaMemcpyHostToDevice,
                           s->target->ctx->stream));
  return alm_spec_begin(s, token, pos);
}

int alm_spec_begin(alm_spec* s, int32_t token, int pos) {
  ALM_REQ(s, "null spec");
  ALM_REQ(token >= 0 && token < s->target->cfg.vocab, "token out of range");
  ALM_REQ(pos >= 0, "negative position");
  ALM_REQ(pos >= 1 || !s->refresh, "the draft refresh needs pos >= 1");
  DeviceGuard g(s->target->ctx->device);
  s->pinned[0] = token;
  s->pinned[1] = pos;
  s->pinned[2] = 0;
  s->pinned[3] = 0;
  cudaStream_t st = s->target->ctx->stream;
  ALM_CUDA(cudaMemcpyAsync(s->state, s->pinned, 4 * sizeof(int), cudaMemcpyHostToDevice, st));
  ALM_CUDA(cudaStreamSynchronize(st));
  return ALM_OK;
}

int alm_spec_state(alm_spec* s, int32_t* token, int32_t* pos) {
  ALM_REQ(s && token && pos, "null argument");
  DeviceGuard g(s->target->ctx->device);
  int st4[4];
  ALM_CUDA(cudaMemcpy(st4, s->state, sizeof(st4), cudaMemcpyDeviceToHost));
  *token = st4[0];
  *pos = st4[1];
  return ALM_OK;
}

// Sampling steps read up to 2k + 1 draws each beyond the cursor.
static int check_uniforms(alm_spec* s, int n_steps) {
  if (!(s->temperature > 0.f)) return ALM_OK;
  int cursor = 0;
  ALM_CUDA(cudaMemcpy(&cursor, s->state + 4, sizeof(int), cudaMemcpyDeviceToHost));
  const long long need = static_cast<long long>(cursor) + static_cast<long long>(n_steps) * (2 * s->k + 1);
  if (need > s->n_uniforms) return fail(ALM_ERR_ARG, "not enough uniform draws loaded (alm_spec_set_uniforms)");
  return ALM_OK;
}

int alm_spec_set_sampling(alm_spec* s, float temperature, float top_p, float min_p) {
  ALM_REQ(s, "null spec");
  ALM_REQ(top_p > 0.f && top_p <= 1.f, "top_p must be in (0, 1]");
  ALM_REQ(min_p >= 0.f && min_p < 1.f, "min_p must be in [0, 1)");
  DeviceGuard g(s->target->ctx->device);
  ALM_CUDA(cudaStreamSynchronize(s->target->ctx->stream));
  s->temperature = temperature > 0.f ? std::max(temperature, 1e-9f) : 0.f;
  s->top_p = top_p;
  s->min_p = min_p;
  return capture_spec_graph(s);
}

int alm_spec_set_draft_refresh(alm_spec* s, int enable) {
  ALM_REQ(s, "null spec");
  DeviceGuard g(s->target->ctx->device);
  ALM_CUDA(cudaStreamSynchronize(s->target->ctx->stream));
  s->refresh = enable != 0;
  return capture_spec_graph(s);
}

int alm_spec_set_rejection(alm_spec* s, int enable) {
  ALM_REQ(s, "null spec");
  DeviceGuard g(s->target->ctx->device);
  ALM_REQ(s->target->cfg.vocab <= kAccMaxChunks * 256, "vocabulary too large for the acceptance kernel");
  ALM_CUDA(cudaStreamSynchronize(s->target->ctx->stream));
  s->rejection = enable != 0;
  return capture_spec_graph(s);
}

int alm_spec_set_uniforms(alm_spec* s, const double* uniforms_host, int n) {
  ALM_REQ(s && (uniforms_host || n == 0), "null argument");
  ALM_REQ(n >= 0, "negative count");
  DeviceGuard g(s->target->ctx->device);
  cudaStream_t st = s->target->ctx->stream;
  ALM_CUDA(cudaStreamSynchronize(st));
  if (n > s->cap_uniforms) {
    dev_free(s->uniforms);
    s->uniforms = nullptr;
    s->cap_uniforms = 0;
    ALM_TRY(dev_alloc_t(&s->uniforms, static_cast<size_t>(n)));
    s->cap_uniforms = n;
    // the captured graph holds the buffer's address
    if (s->temperature > 0.f) ALM_TRY(capture_spec_graph(s));
  }
  if (n) ALM_CUDA(cudaMemcpy(s->uniforms, uniforms_host, static_cast<size_t>(n) * sizeof(double),
                             cudaMemcpyHostToDevice));
  s->n_uniforms = n;
  ALM_CUDA(cudaMemset(s->state + 4, 0, sizeof(int)));
  return ALM_OK;
}

int alm_spec_uniforms_used(alm_spec* s, int32_t* used) {
  ALM_REQ(s && used, "null argument");
  DeviceGuard g(s->target->ctx->device);
  ALM_CUDA(cudaStreamSynchronize(s->target->ctx->stream));
  ALM_CUDA(cudaMemcpy(used, s->state + 4, sizeof(int), cudaMemcpyDeviceToHost));
  return ALM_OK;
}

int alm_spec_run(alm_spec* s, int n_steps, int32_t* emitted_host, int32_t* n_emitted_host,
                 int32_t* accepted_host) {
  ALM_REQ(s && emitted_host && n_emitted_host, "null argument");
  ALM_REQ(n_steps >= 1 && n_steps <= s->cap_steps, "n_steps out of range (1..1024)");
  DeviceGuard g(s->target->ctx->device);
  cudaStream_t st = s->target->ctx->stream;
  int cur[4];
  ALM_CUDA(cudaMemcpy(cur, s->state, sizeof(cur), cudaMemcpyDeviceToHost));
  const int last_pos = cur[1] + n_steps * (s->k + 1) + s->k;
  ALM_REQ(last_pos < s->tkv->max_len && last_pos < s->dkv->max_len, "speculative steps would overflow the kv cache");
  ALM_REQ(last_pos < s->target->cfg.max_len && last_pos < s->draft->cfg.max_len, "position beyond the rope table");
  ALM_TRY(check_uniforms(s, n_steps));
  ALM_CUDA(cudaMemsetAsync(s->state + 2, 0, 2 * sizeof(int), st));
  cudaGraphExec_t graph = step_graph(s, cur[1], n_steps);
  for (int i = 0; i < n_steps; ++i) ALM_CUDA(cudaGraphLaunch(graph, st));
  int* h = s->pinned;
  ALM_CUDA(cudaMemcpyAsync(h, s->state, 4 * sizeof(int), cudaMemcpyDeviceToHost, st));
  ALM_CUDA(cudaStreamSynchronize(st));
  const int n_emit = h[2];
  ALM_CUDA(cudaMemcpyAsync(h + 4, s->out_tokens, n_emit * sizeof(int), cudaMemcpyDeviceToHost, st));
  ALM_CUDA(cudaMemcpyAsync(h + 4 + s->cap_tokens, s->out_acc, n_steps * sizeof(int), cudaMemcpyDeviceToHost, st));
  ALM_CUDA(cudaStreamSynchronize(st));
  std::memcpy(emitted_host, h + 4, n_emit * sizeof(int));
  *n_emitted_host = n_emit;
  if (accepted_host) std::memcpy(accepted_host, h + 4 + s->cap_tokens, n_steps * sizeof(int));
  int err = 0;
  ALM_CUDA(cudaMemcpy(&err, s->target->ws.err, sizeof(int), cudaMemcpyDeviceToHost));
  int err2 = 0;
  ALM_CUDA(cudaMemcpy(&err2, s->draft->ws.err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err == 2 || err2 == 2) return fail(ALM_ERR_CUDA, "a device-side wait gave up (weight stream did not arrive)");
  if (err || err2) return fail(ALM_ERR_TOKEN, "token id outside the vocabulary");
  return ALM_OK;
}

int alm_spec_kernel_count(alm_spec* s, int32_t* n_kernels) {
  ALM_REQ(s && n_kernels, "null argument");
  *n_kernels = s->n_kernels;
  return ALM_OK;
}

int alm_profiler_range(int start) {
  ALM_CUDA(start ? cudaProfilerStart() : cudaProfilerStop());
  return ALM_OK;
}

int alm_spec_bench(alm_spec* s, int n_steps, float* ms, int32_t* n_emitted) {
  ALM_REQ(s && ms && n_emitted, "null argument");
  ALM_REQ(n_steps >= 1 && n_steps <= s->cap_steps, "n_steps out of range (1..1024)");
  DeviceGuard g(s->target->ctx->device);
  cudaStream_t st = s->target->ctx->stream;
  int cur[4];
  ALM_CUDA(cudaMemcpy(cur, s->state, sizeof(cur), cudaMemcpyDeviceToHost));
  const int last_pos = cur[1] + n_steps * (s->k + 1) + s->k;
  ALM_REQ(last_pos < s->tkv->max_len && last_pos < s->dkv->max_len, "speculative steps would overflow the kv cache");
  ALM_TRY(check_uniforms(s, n_steps));
  cudaEvent_t e0, e1;
  ALM_CUDA(cudaEventCreate(&e0));
  ALM_CUDA(cudaEventCreate(&e1));
  ALM_CUDA(cudaMemsetAsync(s->state + 2, 0, 2 * sizeof(int), st));
  cudaGraphExec_t graph = step_graph(s, cur[1], n_steps);
  ALM_CUDA(cudaEventRecord(e0, st));
  for (int i = 0; i < n_steps; ++i) ALM_CUDA(cudaGraphLaunch(graph, st));
  ALM_CUDA(cudaEventRecord(e1, st));
  ALM_CUDA(cudaEventSynchronize(e1));
  ALM_CUDA(cudaEventElapsedTime(ms, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  int st4[4];
  ALM_CUDA(cudaMemcpy(st4, s->state, sizeof(st4), cudaMemcpyDeviceToHost));
  *n_emitted = st4[2];
  return ALM_OK;
}

int alm_spec_profile(alm_spec* s, int cap, int32_t* ops_host, int32_t* rows_host, float* us_host,
                     int32_t* n_out) {
  ALM_REQ(s && ops_host && rows_host && us_host && n_out && cap > 0, "null argument");
  DeviceGuard g(s->target->ctx->device);
  alm_ctx* c = s->target->ctx;
  cudaStream_t st = c->stream;
  int cur[8];
  ALM_CUDA(cudaMemcpy(cur, s->state, sizeof(cur), cudaMemcpyDeviceToHost));
  ALM_REQ(cur[1] + 2 * (s->k + 1) + s->k < s->tkv->max_len && cur[1] + 2 * (s->k + 1) + s->k < s->dkv->max_len,
          "speculative steps would overflow the kv cache");
  ALM_TRY(check_uniforms(s, 1));
  // per-operation launches, no programmatic dependent launch: every kernel
  // runs alone between its two events
  const bool pdl = c->pdl, persist = c->persist;
  c->pdl = false;
  c->persist = false;
  LaunchProfile prof;
  prof.st = st;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int rc = ALM_OK;
  if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    rc = fail(ALM_ERR_CUDA, "graph capture failed to start");
  } else {
    g_prof = &prof;
    prof_mark(ALM_OP_BEGIN, 0);
    // the P.V variant the replayed step graphs would use here
    const bool one_span = step_graph(s, cur[1], 2) != s->graph;
    s->target->pv_one_span = s->draft->pv_one_span = one_span;
    rc = enqueue_spec_step(s);
    s->target->pv_one_span = s->draft->pv_one_span = false;
    g_prof = nullptr;
    const cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (rc == ALM_OK && prof.err != cudaSuccess) rc = fail(ALM_ERR_CUDA, cudaGetErrorString(prof.err));
    if (rc == ALM_OK && e != cudaSuccess) rc = fail(ALM_ERR_CUDA, std::string("capture: ") + cudaGetErrorString(e));
  }
  c->pdl = pdl;
  c->persist = persist;
  if (rc == ALM_OK && cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess)
    rc = fail(ALM_ERR_CUDA, "instantiate of the profiled step failed");
  // two replays (the second one timed), each from the saved state
  for (int rep = 0; rep < 2 && rc == ALM_OK; ++rep) {
    if (cudaMemcpyAsync(s->state, cur, sizeof(cur), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaGraphLaunch(exec, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
      rc = fail(ALM_ERR_CUDA, "replay of the profiled step failed");
  }
  const int n = static_cast<int>(prof.ev.size()) - 1;
  if (rc == ALM_OK && n > cap) rc = fail(ALM_ERR_ARG, "profile capacity too small: " + std::to_string(n) + " launches");
  for (int i = 0; rc == ALM_OK && i < n; ++i) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, prof.ev[i], prof.ev[i + 1]) != cudaSuccess) {
      rc = fail(ALM_ERR_CUDA, "event timing of the profiled step failed");
      break;
    }
    ops_host[i] = prof.op[i + 1];
    rows_host[i] = prof.rows[i + 1];
    us_host[i] = ms * 1000.f;
  }
  if (rc == ALM_OK) *n_out = n;
  cudaMemcpy(s->state, cur, sizeof(cur), cudaMemcpyHostToDevice);
  if (exec) cudaGraphExecDestroy(exec);
  if (graph) cudaGraphDestroy(graph);
  for (cudaEvent_t e : prof.ev) cudaEventDestroy(e);
  return rc;
}

int alm_bench_qmatmul(alm_ctx* ctx, alm_qweight* const* ws, int n_w, const uint16_t* x_dev, int m,
                      uint16_t* y_dev, int iters, float* avg_us) {
  ALM_REQ(ctx && ws && n_w > 0 && x_dev && y_dev && avg_us, "null argument");
  ALM_REQ(iters >= 1, "iters must be positive");
  for (int i = 0; i < n_w; ++i)
    ALM_REQ(ws[i] && ws[i]->out == ws[0]->out && ws[i]->in_real == ws[0]->in_real, "weights must share a shape");
  ALM_REQ(m >= 1 && m <= (ws[0]->t.layout == kLayoutRow ? kMaxDenseRows : kMaxRows),
          "m must be in 1..16 (1..256 for row-layout weights)");
  DeviceGuard g(ctx->device);
  size_t need = 0;
  for (int i = 0; i < n_w; ++i) need = std::max(need, gemv_part_floats(ws[i]->t, m));
  float* part = nullptr;
  if (need) ALM_TRY(dev_alloc_t(&part, need));
  SplitScratch scr{part, need};
  Epi e;
  e.out = reinterpret_cast<half*>(y_dev);
  e.ldo = ws[0]->out;
  e.n_out = ws[0]->out;
  const ActIn in = raw_in(reinterpret_cast<const half*>(x_dev), ws[0]->in_real, ws[0]->in_real);
  // launches are replayed from a CUDA graph (with programmatic dependent
  // launch, as inside a forward) so the host launch rate does not cap them
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int rc = ALM_OK;
  cudaError_t err = cudaEventCreate(&e0);
  if (err == cudaSuccess) err = cudaEventCreate(&e1);
  for (int i = 0; err == cudaSuccess && i < n_w; ++i)   // warm-up
    err = launch_gemv(ws[i]->t, in, m, EPI_STORE, e, StepIO{}, scr, false, ctx->stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(ctx->stream);
  if (err == cudaSuccess) err = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
  if (err == cudaSuccess) {
    cudaError_t le = cudaSuccess;
    for (int i = 0; le == cudaSuccess && i < iters; ++i)
      le = launch_gemv(ws[i % n_w]->t, in, m, EPI_STORE, e, StepIO{}, scr, ctx->pdl, ctx->stream);
    err = cudaStreamEndCapture(ctx->stream, &graph);
    if (err == cudaSuccess) err = le;
  }
  if (err == cudaSuccess) err = cudaGraphInstantiate(&exec, graph, 0);
  if (err == cudaSuccess) err = cudaGraphLaunch(exec, ctx->stream);   // warm replay
  if (err == cudaSuccess) err = cudaEventRecord(e0, ctx->stream);
  if (err == cudaSuccess) err = cudaGraphLaunch(exec, ctx->stream);
  if (err == cudaSuccess) err = cudaEventRecord(e1, ctx->stream);
  if (err == cudaSuccess) err = cudaEventSynchronize(e1);
  float ms = 0.f;
  if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
  if (err != cudaSuccess) rc = fail(ALM_ERR_CUDA, std::string("bench: ") + cudaGetErrorString(err));
  else *avg_us = ms * 1000.f / iters;
  if (exec) cudaGraphExecDestroy(exec);
  if (graph) cudaGraphDestroy(graph);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  dev_free(part);
  return rc;
}

}  // extern "C"

// ---- internal accessors for entry points defined in other files ----------------
int alm_internal_fail(int code, const char* msg) { return fail(code, msg); }

int alm_internal_qweight_tile(const alm_qweight* w, QTile* t, int* out_rows, int* in_real) {
  ALM_REQ(w && t && out_rows && in_real, "null argument");
  *t = w->t;
  *out_rows = w->out;
  *in_real = w->in_real;
  return ALM_OK;
}

int alm_internal_ctx(alm_ctx* ctx, int* device, cudaStream_t* stream) {
  ALM_REQ(ctx && device && stream, "null argument");
  *device = ctx->device;
  *stream = ctx->stream;
  return ALM_OK;
}
