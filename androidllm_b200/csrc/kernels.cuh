// Internal kernel interfaces shared by the .cu files of libandroidllm_b200.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace alm {

// Largest number of activation rows (tokens) one forward processes.
constexpr int kMaxRows = 16;
// Rows of one multi-sequence pass: the GEMV runs more than kMaxRows rows as
// row groups of kMaxRows (one set of CTAs per group, each computing exactly
// what a pass of its rows alone computes).
constexpr int kMaxPassRows = 64;
constexpr int kMaxRowGroups = kMaxPassRows / kMaxRows;
// Attention position chunk and row group.
constexpr int kAttnChunk = 64;
constexpr int kAttnRows = 16;
// Superchunk of positions the P.V kernel stages in shared memory at once.
constexpr int kPvSpan = 1024;
// Query rows per P.V block.  A row's products and sums do not depend on the
// grouping, so this only trades blocks against the exp / divide work of
// forming P in each block: measured on B200 in the benchmark's speculative
// step, 2 rows beat 4 (0.75 %) and 1 (1.7 %).
constexpr int kPvRows = 2;

// ---------------------------------------------------------------------------
// Tiled quantized weight ("qtile" layout).
//
// Rows are grouped in tiles of 16, columns in k-blocks of 64.  Each (tile,
// k-block) is one record: the weight codes followed by their fp16 scales,
// so a warp walks one contiguous stream of records with one pointer bump per
// k-block.  In a record the 32 lanes of a warp hold exactly the m16n8k16 A
// fragments of four k16 steps, so one coalesced 512 B (int4) / 1 KB (int8)
// / 2 KB (fp16) warp load feeds 4 tensor-core MMAs with no shuffles:
//   int4: lane word s (s = k16 step) = nibbles
//         [(g,c) (g+8,c) (g,c+8) (g+8,c+8) (g,c+1) (g+8,c+1) (g,c+9) (g+8,c+9)]
//         with c = 16 s + 2 t, each stored offset-binary (q + 8);
//   int8: lane words 2s, 2s+1 = bytes [(g,c) (g,c+1) (g,c+8) (g,c+9)] and the
//         same for row g+8, offset-binary (q + 128); the two 16 B halves of a
//         lane are stored 512 B apart so each is a coalesced warp load;
//   fp16: lane uint4 s = the four A registers of step s.
// Scales (after the codes): eight half2 {s(g), s(g+8)}, g = 0..7, for the
// record's 64 columns (two such sets for 32-column blocks: steps 0-1 and 2-3).
// Blocks wider than 64 repeat their scale in every record.
// ---------------------------------------------------------------------------
struct QTile {
  const uint4* data = nullptr;   // records, (tile, k-block) major
  int bits = 4;       // 4, 8 or 16 (fp16, no scales)
  int block = 64;     // scale block along K (32 or a multiple of 64)
  int n_rows = 0;     // logical output rows
  int n_tiles = 0;    // ceil(n_rows / 16)
  int k_blocks = 0;   // ceil(k_pad / 64)
  int rec_u4 = 0;     // record size in 16-byte units
  int sb = 0;         // scale sets per record (0 for fp16, 1, or 2 for 32-column blocks)
  int k_real = 0;     // real input length (activation columns)
  // split-K launch shape
  int ksw = 1;        // warps splitting K inside a CTA (1, 2, 4, 8)
  int ksg = 1;        // CTAs splitting K
  int kps = 1;        // k-blocks per split
  unsigned* counters = nullptr;  // one per CTA column, self-resetting
  // record layout: kLayoutTile (above) or kLayoutRow (below)
  int layout = 0;
  int n_rb = 0;       // row layout: 128-row blocks
  int wg = 1;         // row layout: decoding warpgroups per CTA (1, 2, 4)
};

// ---------------------------------------------------------------------------
// Row-record layout ("qrow"), streamed by the tcgen05 GEMV (tc_gemv.cu).
//
// Rows are grouped in blocks of 128 (one tcgen05 MMA tile) and, inside a
// block, in four groups of 32 (one warp, one tensor-memory lane quarter).
// Each (group, k-block of 64) is one record, contiguous along k for a group:
// record index ((rb * 4 + group) * k_blocks + kb).  A record holds, for row t
// of the group, 16-byte parts at p * 512 + t * 16 (so every warp load is
// 512 contiguous bytes), then 32 fp16 scales (row t at 2 t):
//   int4 (2 parts): part p word j = nibbles of k = 32 p + 8 j + (0, 2, 4, 6,
//        1, 3, 5, 7), offset-binary (q + 8): nibbles (0, 4), (1, 5), (2, 6),
//        (3, 7) decode to the fp16 pairs of tensor-memory columns 16 p + 4 j
//        + 0..3 (k pairs (0,1), (2,3), (4,5), (6,7));
//   int8 (4 parts): part p word j = bytes of k = 16 p + 4 j + 0..3,
//        offset-binary (q + 128): columns 8 p + 2 j, 8 p + 2 j + 1.
// Decoding uses the same exact fp16 operations as the tile layout, so both
// layouts dequantize to identical weights.
// ---------------------------------------------------------------------------
constexpr int kLayoutTile = 0;
constexpr int kLayoutRow = 1;
constexpr int kRowBlock = 128;

// An activation operand: either raw fp16 rows, or the un-normalised residual
// sum of the previous layer with its RMSNorm still to apply:
//   x = fp16((f32(v) / sqrt(sum(ss[m, :]) / H + eps)) * f32(w))
// where ss holds per-16-row-tile partial sums of squares written by the
// producing kernel (fixed order, so the result is independent of M).
struct ActIn {
  const half* x = nullptr;
  int ld = 0;
  const float* ss = nullptr;
  int n_ss = 0;
  const half* w = nullptr;
  float eps = 0.f;
  int H = 0;
  int vec = 0;   // rows (and norm weights) allow 16-byte loads; set by the launchers
};

// 16-byte loads are allowed when the base is 16-byte aligned and the row
// stride is a multiple of 8 halves.
__host__ __device__ inline void set_vec(ActIn& a) {
  const bool ok = (reinterpret_cast<uintptr_t>(a.x) % 16 == 0) && (a.ld % 8 == 0) &&
                  (a.w == nullptr || reinterpret_cast<uintptr_t>(a.w) % 16 == 0);
  a.vec = ok ? 1 : 0;
}

enum EpiKind : int { EPI_STORE = 0, EPI_QKV = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_LOGITS = 4, EPI_STORE32 = 5 };

struct Epi {
  half* out = nullptr;   // STORE / RESID / SWIGLU / LOGITS output rows
  float* out32 = nullptr;  // STORE32: fp32 sums before rounding (tensor-parallel partials)
  int ldo = 0;
  int n_out = 0;         // valid output columns (rows of W, or I for SwiGLU)
  // QKV: q (fp32) and the paged K/V cache of one layer
  float* q = nullptr;
  int ldq = 0;
  half* kcache = nullptr;
  half* vcache = nullptr;
  const int* page_table = nullptr;
  int page_size = 16;
  int heads = 0, kv_heads = 0, head_dim = 0;
  const half* rope = nullptr;   // (max_len, head_dim) fp16 [cos | sin]
  // QKV of a multi-sequence pass: per activation row {position, offset of
  // its sequence's row of the page table} (null: pos0 + m, offset 0)
  const int2* rows = nullptr;
  // RESID
  ActIn res;
  float* ss_out = nullptr;      // (M, n_tiles) partial sums of squares
  // LOGITS: per-CTA argmax partials (M, gridDim.x)
  float* am_val = nullptr;
  int* am_idx = nullptr;
};

struct StepIO {
  const int* pos = nullptr;     // device: position of activation row 0
  int* err = nullptr;           // device: set to 2 if a bounded wait gave up
};

// Scratch for cross-CTA split-K partial sums.
struct SplitScratch {
  float* part = nullptr;
  size_t part_floats = 0;
};

// Set per-kernel shared-memory limits on the current device (once per
// device, before any launch or stream capture).
cudaError_t gemv_init_attrs();
cudaError_t attention_init_attrs();
cudaError_t rows_init_attrs();

// launchers (return cudaError_t of the launch)
cudaError_t launch_repack(const void* const* src, const half* const* src_scales, int n_src,
                          const int* dst_src_row, QTile& w, uint4* data, int k_pad, cudaStream_t st);
cudaError_t launch_dequant(const QTile& w, half* out, cudaStream_t st);
cudaError_t launch_gemv(const QTile& w, const ActIn& in, int M, EpiKind kind, const Epi& epi,
                        const StepIO& io, const SplitScratch& scr, bool pdl, cudaStream_t st);
// Row layout: repack, dequantize and the tcgen05 GEMV (tc_gemv.cu).
cudaError_t launch_repack_rows(const void* const* src, const half* const* src_scales, int n_src,
                               const int* dst_src_row, const QTile& w, uint4* data, int k_pad, cudaStream_t st);
cudaError_t launch_dequant_rows(const QTile& w, half* out, cudaStream_t st);
cudaError_t launch_tc_gemv(const QTile& w, const ActIn& in, int M, EpiKind kind, const Epi& epi,
                           const StepIO& io, const SplitScratch& scr, bool pdl, cudaStream_t st);
cudaError_t tc_gemv_init_attrs();
// Dynamic shared memory a row-layout GEMV of `rows` activation rows needs.
size_t tc_gemv_smem_bytes(const QTile& w, int rows);
// Split-K partial floats a GEMV launch of w over `rows` activation rows
// needs (either layout; the row layout's dense path splits K by rows).
size_t gemv_part_floats(const QTile& w, int rows = kMaxRows);
size_t tc_part_floats(const QTile& w, int rows);
// Activation rows one launch takes: 16, or 256 (STORE) for the row layout.
constexpr int kMaxDenseRows = 256;
// CTAs along the output rows (argmax partials of a LOGITS launch).
int gemv_out_blocks(const QTile& w);

// One sequence of a multi-sequence attention pass: activation rows m0 ..
// m0 + n_tok - 1 at positions pos0 .., its pages at page_table + pt_off; its
// scores row groups start at g0 and its P.V groups at p0 (no group holds
// rows of two sequences, so a block reads one sequence's K / V).
struct AttnSeq {
  int m0, n_tok, pos0, pt_off, g0, p0;
};

struct AttnArgs {
  const float* q = nullptr;  int ldq = 0;
  const half* kcache = nullptr;
  const half* vcache = nullptr;
  const int* page_table = nullptr;
  int page_size = 16;
  int heads = 0, kv_heads = 0, head_dim = 0;
  int M = 1;
  const int* pos = nullptr;
  int max_ctx = 0;           // capacity: grid sized for this many positions
  float* scores = nullptr;   // (kv_heads, n_rg, 16, score_ld)
  int score_ld = 0;
  float* stats = nullptr;    // (kv_heads, n_rg, n_chunks_max, 16, 2)
  half* ctx = nullptr;       // (M, heads * head_dim)
  int ldc = 0;
  // P.V split over spans of kPvSplit positions (standalone kernels; null: one
  // block walks every position): fp32 partials of (slice, kv head, row
  // group) per span, and a self-resetting ticket per (slice, kv head, group)
  float* pv_part = nullptr;
  unsigned* pv_ticket = nullptr;
  // multi-sequence pass (null: one sequence of M rows at *pos): the
  // sequences (device, written before the launch) and the pass's total
  // scores row groups and P.V groups
  const AttnSeq* seqs = nullptr;
  int n_seq = 0, n_rg = 0, n_pg = 0;
  // one-launch attention (attn_fused.cu): per (kv head, row group) a count
  // of published chunk statistics and a ticket of finished chunk partials
  // (both self-resetting), the fp32 P.V partials of every chunk, and the
  // word a wait that gives up sets (2)
  unsigned* fz_count = nullptr;
  unsigned* fz_ticket = nullptr;
  float* fz_part = nullptr;
  int* err = nullptr;
};
// Positions one block of the split P.V pass takes (a context longer than one
// split span is spread over blocks), and the split spans of max_ctx positions.
// Measured on B200: splitting at 256 positions made 512-768-position
// contexts slower (more blocks plus the combine), at 1024 it pays from two
// spans on.
constexpr int kPvSplit = kPvSpan;
__host__ __device__ inline int attn_pv_spans(int max_ctx) { return (max_ctx + kPvSplit - 1) / kPvSplit; }
cudaError_t launch_attention(const AttnArgs& a, bool pdl, cudaStream_t st);
// The scores pass alone (scores and chunk statistics).
cudaError_t launch_attention_scores(const AttnArgs& a, bool pdl, cudaStream_t st);
// Scores, then a P.V pass with 16 query rows per block (attn_prefill.cu):
// for passes of many rows (the batched prefill), where V is then read once
// per 16 rows.  Equal to launch_attention up to the fp32 order of the P.V
// sums; page_size >= 16, no split partials.
bool attn_rows16_ok(const AttnArgs& a);
cudaError_t launch_attention_rows16(const AttnArgs& a, bool pdl, cudaStream_t st);
// Attention of a prefill chunk (one sequence): one flash-attention pass
// (online softmax; head_dim 16 / 32 / 64 / 128), else launch_attention_rows16,
// else launch_attention.
bool attn_prefill_flash_ok(const AttnArgs& a);
cudaError_t launch_attention_prefill(const AttnArgs& a, bool pdl, cudaStream_t st);
cudaError_t attn_prefill_init_attrs();
// Scores, statistics and P.V in one launch when the pass's blocks fit on
// the GPU at once (fz_* set); false: the caller runs launch_attention.
bool attn_fused_ok(const AttnArgs& a);
cudaError_t launch_attn_fused(const AttnArgs& a, bool pdl, cudaStream_t st);
cudaError_t attn_fused_init_attrs(int n_sms);
// Single-row decode attention in one kernel (attn_decode.cu), bit-identical
// to launch_attention; attn_decode_ok says whether it takes the shape.
bool attn_decode_ok(const AttnArgs& a);
cudaError_t launch_attn_decode(const AttnArgs& a, bool pdl, cudaStream_t st);
cudaError_t attn_decode_init_attrs();

// ---- speculative rejection sampling (accept.cu) ----------------------------
constexpr int kAccMaxChunks = 4096;   // rows of up to 4096 * 256 entries

// Rows of softmax((l - max) / t), min-p filtered when 0 < min_p < 1.
struct ProbsArgs {
  const half* logits = nullptr;  int ld = 0;
  float* probs = nullptr;        int ldp = 0;
  int vocab = 0;
  float t = 1.f;                 // fp32(max(temperature, 1e-9))
  float min_p = 0.f;
};
// One inverse-CDF draw from a probability row with draw u[*cursor + u_offset].
struct DrawArgs {
  const float* probs = nullptr;
  int vocab = 0;
  const double* u = nullptr;
  const int* cursor = nullptr;   // nullable: 0
  int u_offset = 0;
  int* out = nullptr;
};
// min(1, p/q) acceptance of k candidates; draws u[*cursor + u_offset + i]
// (accept i) and u[*cursor + u_offset + k] (resample).  Outputs: tokens
// (k + 1, the accepted prefix then the resampled / bonus token) and n_acc,
// and, with state, the speculative step's state / ring update.
struct AcceptArgs {
  const float* p = nullptr;  int ldp = 0;
  const float* q = nullptr;  int ldq = 0;
  const int* cand = nullptr;
  int k = 0, vocab = 0;
  const double* u = nullptr;
  const int* cursor = nullptr;
  int u_offset = 0;
  int* tokens = nullptr;
  int* n_acc = nullptr;
  int* state = nullptr;
  int* ring = nullptr;
  int* ring_acc = nullptr;
  int cap_tokens = 0, cap_steps = 0, cursor_advance = 0;
};
cudaError_t launch_probs(const ProbsArgs& a, int rows, cudaStream_t st);
cudaError_t launch_draw(const DrawArgs& a, cudaStream_t st);
cudaError_t launch_accept(const AcceptArgs& a, cudaStream_t st);

// Per-launch profile of a speculative step (alm_spec_profile): while a
// profiled step is being captured, prof_mark records a timing event after
// each kernel launch, tagged with the launch's operation (ALM_OP_* of the
// public header) and activation rows; outside a profiled capture it does
// nothing.
void prof_mark(int op, int rows);

// embedding gather: x0[m] = dequant(embed[token_m])
struct EmbedArgs {
  const void* table = nullptr;   // int4 packed / int8 / fp16 rows
  const half* scale = nullptr;   // (vocab, nsb) or null for fp16
  int bits = 16, block = 0, nsb = 0, hidden = 0, row_bytes = 0, vocab = 0;
  const int* tokens = nullptr;   // (M) device
  half* out = nullptr;           // (M, hidden)
  int M = 1;
  int* err = nullptr;            // set to 1 on an out-of-range token
};
cudaError_t launch_embed(const EmbedArgs& a, bool pdl, cudaStream_t st);

// out[m] = fp16(rmsnorm(x_m)) where x is an ActIn (possibly deferred-norm),
// optionally followed by a second RMSNorm with weight w2 (the final norm).
cudaError_t launch_rownorm(const ActIn& in, int M, const half* w2, float eps2, half* out,
                           int ldo, bool pdl, cudaStream_t st);

// Sampling of rows of fp16 logits (engine.py:26-45 semantics, fixed
// arithmetic; see sample.cu).  Row r draws uniforms[*u_cursor + u_offset + r]
// (u_cursor may be null: 0).  temperature <= 0 gives the argmax.
struct SampleArgs {
  const half* logits = nullptr;
  int ld = 0;
  int vocab = 0;
  float temperature = 0.f;      // max(T, 1e-9) as fp32, or <= 0 for argmax
  float top_p = 1.f;
  float min_p = 0.f;
  const double* uniforms = nullptr;
  const int* u_cursor = nullptr;
  int u_offset = 0;
  float* scratch = nullptr;     // rows * vocab fp32
  int* out = nullptr;           // rows
};
cudaError_t sample_init_attrs();
cudaError_t launch_sample(const SampleArgs& a, int rows, bool pdl, cudaStream_t st);

// argmax over CTA partials -> tokens (M)
cudaError_t launch_argmax_final(const float* am_val, const int* am_idx, int n_part, int M,
                                int* out, bool pdl, cudaStream_t st);

// ---- tensor parallelism (rows.cu) ------------------------------------------
// After the all-reduce of a row-split projection's fp32 partials o32 (M, H):
// out = fp16(res + fp16(o)) with res's deferred norm applied, and per
// 16-column tile sums of squares of out (the RESID epilogue's arithmetic).
cudaError_t launch_tp_resid(const ActIn& res, const float* o32, int M, int H, half* out, float* ss_out, bool pdl,
                            cudaStream_t st);
// Peer-memory all-reduce of a row-split projection (the ranks of one node):
// every rank owns an area of two parity slots x world ranks x rows rows of
// row_floats fp32, then two x world x rows flags; areas[r] is rank r's area
// in this process's address space (its own, or a peer's mapping).
struct TpP2p {
  float* areas[8] = {};
  int world = 0, rank = 0, rows = 0, row_floats = 0;
  unsigned* counters = nullptr;   // this rank's per-row call counts (rows)
  int* err = nullptr;             // set to 2 if a wait gave up
};
constexpr int kTpP2pMaxWorld = 8;
constexpr int kTpP2pHandleBytes = 64;   // a CUDA IPC memory handle
constexpr long long kTpP2pSpinLimit = 1ll << 20;   // polls per peer flag (well under a second)
__host__ __device__ inline size_t tp_p2p_data_floats(int world, int rows, int row_floats) {
  return static_cast<size_t>(2) * world * rows * row_floats;
}
__host__ __device__ inline size_t tp_p2p_area_bytes(int world, int rows, int row_floats) {
  return tp_p2p_data_floats(world, rows, row_floats) * sizeof(float) +
         static_cast<size_t>(2) * world * rows * sizeof(unsigned);
}
__host__ __device__ inline float* tp_p2p_data(const TpP2p& p, float* area, int parity, int src, int m) {
  return area + ((static_cast<size_t>(parity) * p.world + src) * p.rows + m) * p.row_floats;
}
__host__ __device__ inline unsigned* tp_p2p_flag(const TpP2p& p, float* area, int parity, int src, int m) {
  unsigned* flags = reinterpret_cast<unsigned*>(area + tp_p2p_data_floats(p.world, p.rows, p.row_floats));
  return flags + (static_cast<size_t>(parity) * p.world + src) * p.rows + m;
}
cudaError_t launch_tp_p2p_resid(const ActIn& res, const float* o32, int M, int H, half* out, float* ss_out,
                                const TpP2p& p, bool pdl, cudaStream_t st);
// The same with the fp16 outputs of the dense path (batched prefill).
// launch_resid_rows16, then the RMSNorm (nrm: the deferred norm of `out`,
// nrm.ss == ss_out) of the result into xout (row stride ldx), in one kernel.
cudaError_t launch_resid_norm(const ActIn& res, const half* o16, int M, int H, half* out, float* ss_out,
                              const ActIn& nrm, half* xout, int ldx, bool pdl, cudaStream_t st);
cudaError_t launch_resid_rows16(const ActIn& res, const half* o16, int M, int H, half* out, float* ss_out, bool pdl,
                                cudaStream_t st);

// Local argmax of each row from the head GEMV's per-CTA partials, as
// (value bits, global index = local index + offset) pairs.
cudaError_t launch_tp_argmax_local(const float* am_val, const int* am_idx, int n_part, int M, int offset,
                                   int* pairs, bool pdl, cudaStream_t st);
// Best of the all-gathered pairs (world, M, 2) of every row -> out[m].
cudaError_t launch_tp_argmax_pick(const int* pairs, int world, int M, int* out, bool pdl, cudaStream_t st);
// All-gathered local logits (world, M, v_local) -> rows (M, world * v_local).
cudaError_t launch_tp_logits_reorder(const half* gathered, int world, int M, int v_local, half* out, bool pdl,
                                     cudaStream_t st);

// ---- batched prefill (prefill.cu) ------------------------------------------
struct PfRopeArgs {
  const half* qkv = nullptr;   // (M, ld_qkv): q heads, k heads, v heads
  int ld_qkv = 0;
  const half* rope = nullptr;  // (max_len, head_dim) cos | sin
  int pos0 = 0;
  int heads = 0, kv_heads = 0, head_dim = 0;
  float* q = nullptr;          // (M, ldq) fp32 after RoPE
  int ldq = 0;
  half* kcache = nullptr;
  half* vcache = nullptr;
  const int* page_table = nullptr;
  int page_size = 16;
};
cudaError_t launch_pf_rope_kv(const PfRopeArgs& a, int M, bool pdl, cudaStream_t st);
cudaError_t launch_pf_swiglu(const half* gu, int ld_gu, int inter, int M, half* h, int ld_h, bool pdl,
                             cudaStream_t st);

}  // namespace alm
