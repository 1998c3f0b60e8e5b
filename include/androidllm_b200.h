/*
 * libandroidllm_b200 — C ABI of the B200 speculative-decode verify path.
 *
 * The entry points replace androidllm's native kernels and the numpy work of
 * its hot path (paths relative to the androidllm project root):
 *   - src/androidllm_neon.c:71      matmul_f16_f16 (ctypes, androidllm/neon.py:18-51)
 *   - androidllm_rs/src/lib.rs:226  layer_forward  (PyO3, androidllm/models/llama.py:71-94)
 *   - androidllm_rs/src/lib.rs:300  head_logits    (PyO3, androidllm/models/llama.py:130-142)
 *   - androidllm_rs/src/lib.rs:339  sample / androidllm/engine.py:26-61 (greedy pick)
 *   - androidllm/quant.py:58-65     dequantize_packed (per layer per token in engine.py:160-174)
 *   - androidllm/models/llama.py:148-164  prepare_kv
 *   - androidllm/engine.py:288-320  _spec_step (draft K, verify, accept)
 *
 * Conventions: every function returns 0 on success and a nonzero status on
 * error; alm_last_error() then describes the failure (thread-local).  Plain
 * pointers and sizes only.  "_host" arguments are host memory borrowed for the
 * duration of the call; "_dev" arguments are device memory of the context's
 * device.  fp16 data is passed as raw IEEE binary16 (uint16_t).  Each context
 * owns one CUDA stream; calls on one context must not overlap in time.
 */
#ifndef ANDROIDLLM_B200_H
#define ANDROIDLLM_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ALM_API __attribute__((visibility("default")))
#else
#define ALM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct alm_ctx alm_ctx;
typedef struct alm_qweight alm_qweight;
typedef struct alm_model alm_model;
typedef struct alm_kv alm_kv;
typedef struct alm_spec alm_spec;

/* ---- status ---------------------------------------------------------------- */
enum {
  ALM_OK = 0,
  ALM_ERR_ARG = 1,    /* invalid argument (shape, range, null pointer) */
  ALM_ERR_CUDA = 2,   /* CUDA runtime error */
  ALM_ERR_STATE = 3,  /* object not ready (e.g. model layer missing) */
  ALM_ERR_TOKEN = 4   /* a token id outside the vocabulary reached the device */
};

/* Human-readable description of the last error on this thread. */
ALM_API const char* alm_last_error(void);
/* ABI version (major * 100 + minor). */
ALM_API int alm_abi_version(void);

/* ---- context ---------------------------------------------------------------- */
/* Create a context (device + stream). */
ALM_API int alm_ctx_create(int device, alm_ctx** out);
ALM_API int alm_ctx_destroy(alm_ctx* ctx);
ALM_API int alm_ctx_sync(alm_ctx* ctx);
/* Forwards of up to 8 rows as one persistent kernel (enable = 1) or as one
   launch per layer operation (enable = 0, the default; the environment
   variable ALM_PERSIST=1 turns the persistent kernel on at context creation).
   The results are bit-identical.  Graphs captured earlier keep their kernels. */
ALM_API int alm_ctx_set_persistent(alm_ctx* ctx, int enable);
/* Single-row forwards (decode steps, the speculative draft) of models whose
   projections fit it run the embedding and every layer as one launch of one
   16-CTA thread-block cluster (enable = 1; ALM_CLUSTER=1 at context creation
   turns it on), or as one launch per layer operation (enable = 0, the
   default).  The results are bit-identical.  Measured on B200 at the
   Qwen2.5-0.5B draft shape it is slower (2.8 ms against 0.87 ms per
   forward): 16 SMs cannot decode int4 weights as fast as the whole GPU.
   Graphs captured earlier keep their kernels. */
/* Attention of decode / verify passes as one launch (scores, statistics and
 * P.V; the probabilities are the two passes' bit for bit, the P.V sums are
 * added per 64-position chunk and then across chunks) when the pass's blocks
 * fit on the GPU at once, else the two passes (opt-in, default off;
 * ALM_ATTN_FUSED=1 turns the default on).  Measured slower on B200 than the
 * two passes at the benchmark's shapes; passes of different grid sizes may
 * take different paths, so results are bit-equal across passes only at
 * settings where both take the same one. */
ALM_API int alm_ctx_set_attn_fused(alm_ctx* ctx, int enable);
ALM_API int alm_ctx_set_cluster_forward(alm_ctx* ctx, int enable);
/* Weight layout chosen by later uploads: 0 (the default) = 16-row tiles for
   the mma.sync GEMV; 1 = 128-row records for the tcgen05 kernel for weights of
   at least 4 MB, tiles otherwise; 2 = 128-row records wherever the format
   allows (int4 / int8, 64-column blocks; never the fused QKV projection).
   ALM_TC=0/1/2 sets it at context creation.  Dequantized weights are
   identical in both layouts; GEMV results agree to fp32 summation order.
   On B200 a tcgen05.mma costs about the same for N = 16 as for N = 256, so
   the row layout pays off only for many activation rows (dense GEMM). */
ALM_API int alm_ctx_set_gemv_layout(alm_ctx* ctx, int mode);
/* Tensor parallelism (larger models split over the GPUs of one node; no
 * reference counterpart, the reference runs whole matrices in one
 * process, androidllm/models/llama.py:97-127).  One process per GPU; rank 0
 * makes an NCCL unique id (128 bytes) that the host hands to every rank,
 * and each rank joins with alm_ctx_init_tp on its context.  NCCL is opened
 * at run time (libnccl.so.2); the collectives run on the context's stream. */
ALM_API int alm_nccl_unique_id(uint8_t* id_out);
ALM_API int alm_ctx_init_tp(alm_ctx* ctx, int rank, int world, const uint8_t* id);
/* Device memory helpers for hosts without their own device-memory library. */
ALM_API int alm_dev_alloc(alm_ctx* ctx, size_t bytes, void** out_dev);
ALM_API int alm_dev_free(alm_ctx* ctx, void* dev);
ALM_API int alm_copy_h2d(alm_ctx* ctx, void* dst_dev, const void* src_host, size_t bytes);
ALM_API int alm_copy_d2h(alm_ctx* ctx, void* dst_host, const void* src_dev, size_t bytes);

/* ---- quantized weights (androidllm/quant.py format) --------------------------- */
/* Upload one projection in the shard format (androidllm/shard.py:109-120):
 *   bits 4: packed (out, in/2) uint8, even column in the low nibble;
 *   bits 8: (out, in) int8;   bits 16: (out, in) fp16, scale_host NULL.
 *   scale_host: (out, in/block) fp16.  `in` is the stored (padded) input dim,
 *   `in_real` the real one (manifest "in_real").  The weight is repacked on
 *   the device into the tensor-core tile layout.                              */
ALM_API int alm_qweight_upload(alm_ctx* ctx, const void* packed_host, const void* scale_host, int bits,
                       int block, int out, int in, int in_real, alm_qweight** w);
ALM_API int alm_qweight_free(alm_qweight* w);
/* Launch shape of the weight's GEMV: ksw warps split K inside a CTA (1, 2, 4
 * or 8), ksg CTAs split it further (tuning; the default is chosen at upload).
 * A weight already inside a model must not be changed while a forward runs. */
ALM_API int alm_qweight_set_split(alm_qweight* w, int ksw, int ksg);
ALM_API int alm_qweight_get_split(const alm_qweight* w, int* ksw, int* ksg, int* kps);
/* Replaces androidllm/quant.py:58-65 dequantize_packed (sliced to in_real):
 * writes fp16 (out, in_real) to out_host; bit-exact. */
ALM_API int alm_qweight_dequant(alm_ctx* ctx, const alm_qweight* w, uint16_t* out_host);
/* y(m, out) = fp16(x(m, in_real) . W^T), fp32 accumulation, 1 <= m <= 16
   (1 <= m <= 256 for a weight in the row layout: tcgen05 MMAs with N = m).
 * Device buffers; row strides in elements. */
ALM_API int alm_qmatmul(alm_ctx* ctx, const alm_qweight* w, const uint16_t* x_dev, int ldx, int m,
                uint16_t* y_dev, int ldy);
/* alm_qmatmul without any device allocation.  No counterpart in the
 * reference (its CPU kernels never allocate device memory).  For callers that
 * cannot call cudaMalloc once running: real-time loops that cannot take the
 * implicit synchronisation of cudaMalloc/cudaFree, and hosts that reserve
 * their device memory up front and forbid later driver allocations.  The
 * split-K scratch is a fixed array inside the library (2 MiB of partial sums
 * + 4096 counters, held by every GPU that loads the library until exit);
 * weights whose split needs more are rejected with ALM_ERR_ARG.  The first
 * call on a device resolves the array's address (cudaGetSymbolAddress) and
 * should come before any stream capture.  All calls on a device share the
 * array, so calls that overlap on the GPU race; the counters are cleared at
 * the start of each call. */
ALM_API int alm_qmatmul_noalloc(alm_ctx* ctx, const alm_qweight* w, const uint16_t* x_dev, int ldx, int m,
                                uint16_t* y_dev, int ldy);
/* Replaces src/androidllm_neon.c:71 matmul_f16_f16 (out = a . b^T, raw fp16,
 * host buffers, m <= 16): the weight b is uploaded per call. */
ALM_API int alm_matmul_f16_f16(alm_ctx* ctx, const uint16_t* a_host, const uint16_t* b_host,
                       uint16_t* out_host, int m, int k, int n);

/* ---- model ------------------------------------------------------------------- */
/* androidllm canon config (androidllm/config.py:34-48). */
typedef struct alm_model_config {
  int hidden, layers, heads, kv_heads, head_dim, intermediate, vocab;
  int max_len;          /* rows of the RoPE table */
  float rms_eps;
} alm_model_config;

/* One projection in shard format (see alm_qweight_upload). */
typedef struct alm_proj_src {
  const void* packed_host;
  const void* scale_host;
  int bits, block, out, in, in_real;
} alm_proj_src;

/* rope_host: (max_len, head_dim) fp16 [cos | sin] table, androidllm/models/llama.py:27-31. */
ALM_API int alm_model_create(alm_ctx* ctx, const alm_model_config* cfg, const uint16_t* rope_host,
                     alm_model** out);
ALM_API int alm_model_destroy(alm_model* m);
/* proj: 7 entries in the order q, k, v, o, gate, up, down (shard.py:111 bases);
 * n_in / n_post: (hidden) fp16 input_layernorm / post_attention_layernorm. */
ALM_API int alm_model_set_layer(alm_model* m, int layer, const alm_proj_src* proj, const uint16_t* n_in_host,
                        const uint16_t* n_post_host);
/* Embedding rows (vocab, hidden): bits 16 = fp16 table (scale NULL), or the
 * shard's quantized embedding (embed.q / embed.scale with its block). */
ALM_API int alm_model_set_embed(alm_model* m, const void* table_host, const void* scale_host, int bits, int block);
/* Final norm (hidden) fp16. */
ALM_API int alm_model_set_final_norm(alm_model* m, const uint16_t* w_host);
/* Untied LM head (vocab, hidden) in shard format; without it the head is the
 * embedding table (tied, androidllm/models/llama.py:145). */
ALM_API int alm_model_set_head(alm_model* m, const alm_proj_src* head);
/* Make the model this rank's tensor-parallel shard (before set_head and
 * finalize; the context must have joined with alm_ctx_init_tp).  The
 * model's config then holds the rank's heads, kv heads and FFN width, and
 * its layers the matching slices: q / k / v and gate / up rows of its heads
 * and FFN columns, o and down columns (K) of the same, on 64-column blocks.
 * The head is this rank's vocabulary rows [vocab_offset, vocab_offset +
 * vocab_local) with vocab_local * world == vocab (alm_model_set_head; the
 * embedding stays whole).  After the o and down projections the fp32 partial
 * sums are summed over the ranks (ncclAllReduce), then rounded to fp16 and
 * added to the residual; the head's per-rank (max, index) pairs are gathered
 * (ncclAllGather) and the best taken, first index on ties, so every rank
 * holds the same tokens.  Logits requested by the host (or the sampler) are
 * gathered whole. */
ALM_API int alm_model_set_tp(alm_model* m, int vocab_offset, int vocab_local);
/* Peer-memory all-reduce for the row-split projections (o, down) in place of
 * NCCL: each rank opens a receive area sized for rows of row_floats fp32 (the
 * model's hidden size) and gets its CUDA IPC handle (64 bytes) in
 * handle_out; once every rank has every handle (world x 64 bytes in rank
 * order), alm_tp_p2p_connect maps the peers' areas.  A row-split projection
 * then runs its GEMV and one kernel that writes each row to every peer,
 * waits for theirs (bounded) and adds the ranks in rank order — the same sum
 * on every rank — before the residual.  Every rank must connect before any
 * forward; no multicast is used. */
ALM_API int alm_tp_p2p_open(alm_ctx* ctx, int row_floats, uint8_t* handle_out);
ALM_API int alm_tp_p2p_connect(alm_ctx* ctx, const uint8_t* handles);
/* Use the peer all-reduce (1, after connecting) or NCCL (0). */
ALM_API int alm_ctx_set_tp_p2p(alm_ctx* ctx, int enable);
/* *uses_cluster = 1 when the model's single-row forwards run as the cluster
   kernel (alm_ctx_set_cluster_forward enabled and every projection fits it). */
ALM_API int alm_model_cluster_forward(const alm_model* m, int* uses_cluster);
/* Validate and allocate work buffers; required before any forward. */
ALM_API int alm_model_finalize(alm_model* m);

/* ---- paged KV cache (replaces androidllm/models/llama.py:148-164 prepare_kv) -- */
/* fp16 K and V for every layer, `max_len` positions in pages of page_size
 * positions (identity page table, zero-initialised). */
ALM_API int alm_kv_create(alm_ctx* ctx, const alm_model* m, int max_len, int page_size, alm_kv** out);
ALM_API int alm_kv_destroy(alm_kv* kv);
ALM_API int alm_kv_zero(alm_kv* kv);
/* Copy positions [pos0, pos0+n) of one layer out as (n, kv_heads, head_dim)
 * fp16 K and V (the reference cache layout); either pointer may be NULL. */
ALM_API int alm_kv_read(alm_kv* kv, int layer, int pos0, int n, uint16_t* k_host, uint16_t* v_host);
/* Copy (n, kv_heads, head_dim) fp16 rows into the cache at [pos0, pos0+n). */
ALM_API int alm_kv_write(alm_kv* kv, int layer, int pos0, int n, const uint16_t* k_host, const uint16_t* v_host);
/* A cache of n_slots sequences (one per concurrent session of
 * androidllm/batching.py:32-149) of max_len positions each, in pages of
 * page_size positions; slot s starts on pages s * ceil(max_len / page_size)..
 * Single-sequence calls use slot 0. */
ALM_API int alm_kv_create_slots(alm_ctx* ctx, const alm_model* m, int n_slots, int max_len, int page_size,
                                alm_kv** out);
/* alm_kv_read of slot `slot`. */
ALM_API int alm_kv_read_slot(alm_kv* kv, int slot, int layer, int pos0, int n, uint16_t* k_host, uint16_t* v_host);
/* Map the first n pages of slot `slot` to physical pages pages_host[0..n) of
 * the cache (any of its n_slots * pages-per-slot pages). */
ALM_API int alm_kv_set_pages(alm_kv* kv, int slot, const int32_t* pages_host, int n);

/* ---- forward ------------------------------------------------------------------ */
/* Replaces androidllm_rs/src/lib.rs:226 layer_forward (and llama.py:96-128):
 * one post-norm decoder layer over m consecutive positions pos0..pos0+m-1
 * (m = 1 for a decode step, m = k+1 for a verify pass); writes K/V at those
 * positions; x_host, out_host: (m, hidden) fp16. */
ALM_API int alm_layer_forward(alm_model* m, int layer, alm_kv* kv, const uint16_t* x_host, int rows, int pos0,
                      uint16_t* out_host);
/* Replaces androidllm_rs/src/lib.rs:300 head_logits (llama.py:130-146):
 * logits of hidden states x (rows, hidden): fp16-rounded values as fp32
 * (rows, vocab); argmax_host (rows) gets the first maximal index.  Either
 * output may be NULL. */
ALM_API int alm_head_logits(alm_model* m, const uint16_t* x_host, int rows, float* logits_host,
                    int32_t* argmax_host);
/* Replaces androidllm_rs/src/lib.rs:339 sample and androidllm/engine.py:26-45
 * _sample for `rows` rows of fp16 logits (rows, vocab): temperature <= 0 gives
 * the argmax (first index); otherwise softmax(l / T), the min-p filter when
 * 0 < min_p < 1, the top-p nucleus when top_p < 1, then the inverse CDF at
 * the caller's uniform draw uniforms_host[r] in [0, 1) (the draw numpy's
 * Generator.choice takes; the Rust sampler's seed has no counterpart).  The
 * arithmetic is fixed (reproducible exp, fixed-order sums, exact integer
 * cumulative masses, ties in the nucleus by ascending index), so results
 * are deterministic. */
ALM_API int alm_sample(alm_ctx* ctx, const uint16_t* logits_host, int rows, int vocab, float temperature,
                 float top_p, float min_p, const double* uniforms_host, int32_t* out_host);
/* softmax(l / T) of rows of fp16 logits (rows, vocab) -> fp32 probs_host,
 * min-p filtered when 0 < min_p < 1, with fixed arithmetic (rexp, sums in
 * 256-element chunks, sequential) so results are reproducible bit for bit.
 * The distribution the rejection sampler works on (no reference counterpart;
 * the reference's engine.py:29-36 computes the same softmax in numpy). */
ALM_API int alm_probs(alm_ctx* ctx, const uint16_t* logits_host, int rows, int vocab, float temperature, float min_p,
                      float* probs_host);
/* Speculative rejection sampling of k draft candidates (the accept(...)
 * entry of the verify path's boundary; no reference counterpart, the reference accepts by its own rule,
 * engine.py:306-320): p = alm_probs of the k + 1 target logit rows
 * target_logits_host (k + 1, vocab), q = draft_probs_host (k, vocab) the
 * distributions the candidates draft_tokens_host (k) were drawn from.
 * Candidate i is accepted iff fp32(uniforms[i]) * q_i(x_i) < p_i(x_i); at the
 * first rejection the token is drawn from max(0, p_i - q_i) (or p_i if that
 * has no positive entry) by inverse CDF at uniforms[k]; after k accepts the
 * bonus token is drawn from p_k the same way.  out_tokens_host (capacity
 * k + 1) receives the accepted candidates and the drawn token,
 * *n_accepted_host the number accepted (tokens emitted = n + 1). */
ALM_API int alm_accept(alm_ctx* ctx, const uint16_t* target_logits_host, const float* draft_probs_host,
                       const int32_t* draft_tokens_host, int k, int vocab, float temperature, float min_p,
                       const double* uniforms_host, int32_t* out_tokens_host, int32_t* n_accepted_host);
/* alm_sample on the first `rows` rows of the model's last computed logits
 * (alm_forward with a head) without copying them to the host. */
ALM_API int alm_model_sample(alm_model* m, int rows, float temperature, float top_p, float min_p,
                       const double* uniforms_host, int32_t* out_host);
/* alm_model_sample on rows row0 .. row0 + rows - 1 (row0 + rows <= 64) of
 * the last logits (one sequence of a multi-sequence pass). */
ALM_API int alm_model_sample_rows(alm_model* m, int row0, int rows, float temperature, float top_p, float min_p,
                                  const double* uniforms_host, int32_t* out_host);
/* Embedding + every layer + final norm + head for tokens at positions
 * pos0..pos0+rows-1 (androidllm/engine.py:255-286 without sampling). */
ALM_API int alm_forward(alm_model* m, alm_kv* kv, const int32_t* tokens_host, int rows, int pos0,
                float* logits_host, int32_t* argmax_host);
/* Several sequences in one forward (batched sessions; the reference steps
 * them one at a time, androidllm/batching.py:200-272): sequence s has
 * n_tok[s] consecutive rows of tokens_host at positions pos0[s].. of KV slot
 * slots[s] (at most 16 sequences in distinct slots, at most
 * alm_model_max_pass_rows rows in all).  Logits / argmax rows follow
 * tokens_host; each equals its sequence's own alm_forward. */
ALM_API int alm_forward_seqs(alm_model* m, alm_kv* kv, int n_seq, const int32_t* slots, const int32_t* n_tok,
                             const int32_t* pos0, const int32_t* tokens_host, float* logits_host,
                             int32_t* argmax_host);
/* *rows = the most rows one alm_forward_seqs pass takes: 64 (the weights
 * stream once per pass, 16-row groups each computing what a pass of their
 * rows alone computes), 16 on a context with tcgen05 decode weights, 0 for
 * a tensor-parallel model (no multi-sequence passes). */
ALM_API int alm_model_max_pass_rows(const alm_model* m, int* rows);
/* Prompt prefill: fills the KV cache for positions pos0..pos0+n-1 from the
 * tokens, no logits.  Replaces the per-token forwards of the prompt in
 * androidllm/engine.py:345-361.  Chunks of up to 256 rows run every
 * projection through the dense tcgen05 path when the model keeps row-layout
 * copies (alm_model_dense_prefill), the rest in forwards of up to 16 rows. */
ALM_API int alm_prefill(alm_model* m, alm_kv* kv, const int32_t* tokens_host, int n, int pos0);
/* alm_prefill into KV slot `slot` (alm_kv_create_slots). */
ALM_API int alm_prefill_slot(alm_model* m, alm_kv* kv, int slot, const int32_t* tokens_host, int n, int pos0);
/* Whether models created on this context from now on keep row-layout copies
 * of their int4 / int8 (64-column block) projections for alm_prefill
 * (default on; ALM_DENSE_PREFILL=0 turns the default off).  The copies take
 * as much device memory as the layers' weights. */
ALM_API int alm_ctx_set_dense_prefill(alm_ctx* ctx, int enable);
/* *dense = 1 when every layer of the model has its row-layout copies. */
ALM_API int alm_model_dense_prefill(const alm_model* m, int* dense);
/* Profiling (no counterpart in the reference): alm_forward with the head,
 * run as the persistent forward kernel (rows <= 8), recording global-timer
 * nanoseconds; for rows = 1 of a model on the cluster forward, the cluster
 * kernel alone, with *n_ctas = 1: trace_host[0] = n, then n points of CTA 0's
 * decoding threads (label << 48 | global-timer ns: 1 phase start, 2 input
 * staged, 3 first warp's items done, 4 all items done, 5 epilogue done,
 * 6 phase sync passed, 7 scores done, 8 P.V done), and from cap / 2 the
 * same for its weight producer (16 + p / 32 + p: first / last chunk of
 * projection p issued).  trace_host receives n_barriers * n_ctas arrival times
 * (barrier-major: when each CTA finished a phase) followed by n_barriers
 * times at which CTA 0 passed each barrier; cap is its length in entries.
 * Fails with ALM_ERR_STATE when the persistent kernel is unavailable. */
ALM_API int alm_forward_trace(alm_model* m, alm_kv* kv, const int32_t* tokens_host, int rows, int pos0,
                      uint64_t* trace_host, int cap, int* n_barriers, int* n_ctas);

/* ---- speculative decoding (androidllm/engine.py:288-320) ----------------------- */
/* A greedy speculative decoder: K draft steps (M = 1 forwards of `draft`)
 * then one (K+1)-row verify forward of `target` and the acceptance, all on
 * the device and replayed as one CUDA graph per step.  Greedy rule of
 * engine.py:306-320: accept while the target's pick equals the candidate,
 * then emit the target's correction (or the bonus token after K accepts). */
ALM_API int alm_spec_create(alm_model* target, alm_model* draft, alm_kv* target_kv, alm_kv* draft_kv, int k,
                    alm_spec** out);
ALM_API int alm_spec_destroy(alm_spec* s);
/* Set the step state: `token` is the id at position `pos` (the prompt's last
 * token after prefill, engine.py:353-354). */
ALM_API int alm_spec_begin(alm_spec* s, int32_t token, int pos);
/* Run n_steps speculative steps back to back on the device.  emitted_host
 * receives the emitted tokens in order (capacity n_steps * (k+1)),
 * n_emitted_host their count, accepted_host (optional, n_steps) the number
 * of accepted draft tokens of each step.  The state advances. */
ALM_API int alm_spec_run(alm_spec* s, int n_steps, int32_t* emitted_host, int32_t* n_emitted_host,
                 int32_t* accepted_host);
/* alm_spec_begin that also sets the token at pos - 1, which the draft
 * refresh (alm_spec_set_draft_refresh) forwards again; steps keep it up to
 * date themselves, and alm_spec_begin leaves the last step's value. */
ALM_API int alm_spec_begin_prev(alm_spec* s, int32_t prev_token, int32_t token, int pos);
/* Current (token, pos) state. */
ALM_API int alm_spec_state(alm_spec* s, int32_t* token, int32_t* pos);
/* Number of kernel nodes in one speculative step's CUDA graph. */
ALM_API int alm_spec_kernel_count(alm_spec* s, int32_t* n_kernels);
/* Sampling steps (engine.py:296-320 at temperature > 0): every draft
 * candidate is the draft's sample and every verify row the target's sample
 * (alm_sample's rule), accepted while they agree.  temperature <= 0 restores
 * the greedy step.  Re-captures the step graph. */
ALM_API int alm_spec_set_sampling(alm_spec* s, float temperature, float top_p, float min_p);
/* Draft refresh (no reference counterpart; a fix of the reference's draft
 * side, androidllm/engine.py:299-303 vs 318-320): after a step that accepts
 * all k candidates the reference's draft never forwards the last one, so its
 * cache holds a stale entry at that position.  With enable = 1 the first draft
 * forward of every step runs two rows, the token at pos - 1 again and the
 * state token, which rewrites that entry (or recomputes the same values when
 * it was already right).  Emitted tokens do not change (the target verifies
 * every candidate); acceptance can only rise.  Off by default (the reference's
 * behaviour).  Needs pos >= 1.  Re-captures the step graph. */
ALM_API int alm_spec_set_draft_refresh(alm_spec* s, int enable);
/* Sampling steps with min(1, p/q) rejection sampling (enable = 1) instead
 * of the reference's rule (engine.py:306-320, the default): each draft
 * candidate is drawn from the draft's softmax(l / T) row (min-p filtered;
 * top-p is not applied in this mode, since the rule needs the distributions
 * the candidates were drawn from), candidate i is accepted iff
 * u_i * q_i(x) < p_i(x), the first rejected row is resampled from
 * max(0, p - q), and after k accepts a bonus token is drawn from the last
 * target row.  A step consumes exactly 2k + 1 draws: k candidate draws, k
 * acceptance draws, one resample draw.  No reference counterpart: the
 * reference has no rejection sampler.  Re-captures the step graph. */
ALM_API int alm_spec_set_rejection(alm_spec* s, int enable);
/* Load the stream of uniform draws in [0, 1) the sampling steps consume in
 * the reference's order (the k draft samples, then one per target row up to
 * the first rejection); resets the cursor to the stream's start.  A run of n
 * steps needs cursor + n * (2k + 1) draws loaded. */
ALM_API int alm_spec_set_uniforms(alm_spec* s, const double* uniforms_host, int n);
/* Draws of the loaded stream consumed so far. */
ALM_API int alm_spec_uniforms_used(alm_spec* s, int32_t* used);

/* ---- measurement ---------------------------------------------------------------- */
/* Replay n_steps speculative steps back to back and time them with CUDA
 * events on the context's stream: *ms = device time, *n_emitted = tokens.
 * The state advances as in alm_spec_run. */
ALM_API int alm_spec_bench(alm_spec* s, int n_steps, float* ms, int32_t* n_emitted);
/* Operations of a speculative step, as alm_spec_profile reports them
 * (op + 100 * role; role 1 = draft forward, 2 = target verify forward,
 * 0 = the step's own bookkeeping). */
enum {
  ALM_OP_BEGIN = 0, ALM_OP_EMBED = 1, ALM_OP_QKV = 2, ALM_OP_ATTN_SCORES = 3, ALM_OP_ATTN_PV = 4,
  ALM_OP_O = 5, ALM_OP_GATE_UP = 6, ALM_OP_DOWN = 7, ALM_OP_FINAL_NORM = 8, ALM_OP_HEAD = 9,
  ALM_OP_ARGMAX = 10, ALM_OP_SPEC_PREP = 11, ALM_OP_SPEC_ACCEPT = 12, ALM_OP_SAMPLE = 13,
  ALM_OP_LAYERS = 14,  /* embedding and every layer as one cluster kernel */
  ALM_OP_ATTN = 15     /* attention as one launch (alm_ctx_set_attn_fused, or the opt-in single-row kernel) */
};
/* Device time of every kernel launch of one speculative step (profiling; no
 * counterpart in the reference).  The step is captured once more with a
 * timing event after each launch and without programmatic dependent launch,
 * replayed from the current state (which is restored afterwards), and
 * timed on the context's stream: launch i ran from event i to event i+1.
 * ops_host / rows_host / us_host (capacity cap) receive each launch's
 * operation code (see above), activation rows and microseconds; *n_out
 * their count.  Kernels back to back without overlap: the shares, not the
 * sum, are what compare with the step graph. */
ALM_API int alm_spec_profile(alm_spec* s, int cap, int32_t* ops_host, int32_t* rows_host, float* us_host,
                             int32_t* n_out);
/* Start (1) or stop (0) the CUDA profiler's capture range, so a profiler
 * started with capture disabled records only the work in between. */
ALM_API int alm_profiler_range(int start);
/* Time `iters` launches of the dequant-GEMV (x_dev: m rows) cycling through
 * n_w weights of one shape (so their total can exceed L2); *avg_us is the
 * mean device time of one launch. */
ALM_API int alm_bench_qmatmul(alm_ctx* ctx, alm_qweight* const* ws, int n_w, const uint16_t* x_dev, int m,
                              uint16_t* y_dev, int iters, float* avg_us);

#ifdef __cplusplus
}
#endif
#endif /* ANDROIDLLM_B200_H */
