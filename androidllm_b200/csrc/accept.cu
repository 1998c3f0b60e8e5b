// Speculative rejection sampling on the device: min(1, p/q) acceptance of
// the draft's candidates, the residual max(0, p - q) resample at the first
// rejection (or a bonus draw from the last target row), and the accepted
// prefix length from one warp ballot.  This is the acceptance rule of
// speculative sampling, offered beside the reference's own rule (accept while
// an independent target sample equals the draft sample,
// androidllm/engine.py:306-320), which stays the default.
//
// The arithmetic is fixed so it can be restated bit for bit on the CPU:
//   * probabilities: softmax((l - max) / T) with rexp, a total summed in
//     chunks of 256 consecutive elements (sequential inside a chunk, then
//     sequential over the chunk totals), p = e / total; with 0 < min_p < 1,
//     entries below fp32(min_p) * max(p) are zeroed and the row renormalised
//     the same way;
//   * candidate i is accepted iff fp32(u_i) * q_i[x_i] < p_i[x_i] (one fp32
//     product: u < min(1, p/q) for q > 0);
//   * inverse CDF: target = fp32(u) * total; walk the running sum of the
//     chunk totals to the first chunk where it exceeds the target (or the
//     last chunk), then the running sum of that chunk's elements to the first
//     positive element where it exceeds the target; fall back to the chunk's
//     last positive element, then the row's.
// Every sum is one thread's sequential fp32 adds (__fadd_rn), every product,
// quotient and difference one correctly rounded fp32 operation.
#include "common.cuh"
#include "kernels.cuh"

namespace alm {
namespace {

constexpr int kAccThreads = 1024;
constexpr int kAccWarps = kAccThreads / kWarp;
constexpr int kChunk = 256;

struct AccShared {
  float cs[kAccMaxChunks];
  float redf[kAccWarps];
  int redi[kAccWarps];
  float bc_f;
  int bc_i;
  int n_acc;
  int cursor;
  int use_p;     // residual had no positive entry: resample the target row
};

ALM_DEV float block_max(float v, AccShared& sh) {
  v = warp_max(v);
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  if (lane == 0) sh.redf[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < kAccWarps ? sh.redf[lane] : kNegInf;
    w = warp_max(w);
    if (lane == 0) sh.bc_f = w;
  }
  __syncthreads();
  const float r = sh.bc_f;
  __syncthreads();
  return r;
}

ALM_DEV int block_max_int(int v, AccShared& sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  if (lane == 0) sh.redi[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kAccWarps ? sh.redi[lane] : -1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = max(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (lane == 0) sh.bc_i = w;
  }
  __syncthreads();
  const int r = sh.bc_i;
  __syncthreads();
  return r;
}

// A row the walk reads: plain probabilities, or the residual max(0, p - q).
struct RowVec {
  const float* p = nullptr;
  const float* q = nullptr;   // non-null: residual
  ALM_DEV float operator()(int j) const {
    if (!q) return p[j];
    return fmaxf(fsub(p[j], q[j]), 0.f);
  }
};

// sh.cs[c] = sequential fp32 sum of chunk c; returns the sequential total
// (every thread gets it).
template <typename V>
ALM_DEV float chunk_total(const V& v, int n, AccShared& sh) {
  const int n_chunk = (n + kChunk - 1) / kChunk;
  for (int c = threadIdx.x; c < n_chunk; c += kAccThreads) {
    const int lo = c * kChunk, hi = min(lo + kChunk, n);
    float acc = 0.f;
    for (int j = lo; j < hi; ++j) acc = fadd(acc, v(j));
    sh.cs[c] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int c = 0; c < n_chunk; ++c) t = fadd(t, sh.cs[c]);
    sh.bc_f = t;
  }
  __syncthreads();
  const float t = sh.bc_f;
  __syncthreads();
  return t;
}

// Inverse CDF of row v at draw u (see the header comment); every thread
// returns the index.  Precondition: the row has a positive entry.
template <typename V>
ALM_DEV int walk_row(const V& v, int n, double u, AccShared& sh) {
  int last_pos = -1;
  for (int j = threadIdx.x; j < n; j += kAccThreads)
    if (v(j) > 0.f) last_pos = j;
  const int row_last = block_max_int(last_pos, sh);
  const float total = chunk_total(v, n, sh);
  if (threadIdx.x == 0) {
    const int n_chunk = (n + kChunk - 1) / kChunk;
    const float target = fmul(__double2float_rn(u), total);
    float acc = 0.f;
    int c = 0;
    for (; c < n_chunk; ++c) {
      const float nxt = fadd(acc, sh.cs[c]);
      if (nxt > target || c == n_chunk - 1) break;
      acc = nxt;
    }
    const int lo = c * kChunk, hi = min(lo + kChunk, n);
    int pick = -1, chunk_last = -1;
    for (int j = lo; j < hi; ++j) {
      const float x = v(j);
      if (x > 0.f) chunk_last = j;
      acc = fadd(acc, x);
      if (acc > target && x > 0.f) {
        pick = j;
        break;
      }
    }
    if (pick < 0) pick = chunk_last >= 0 ? chunk_last : row_last;
    sh.bc_i = pick;
  }
  __syncthreads();
  const int r = sh.bc_i;
  __syncthreads();
  return r;
}

// Rows of softmax((l - max) / t) (with the min-p filter when 0 < min_p < 1),
// one CTA per row.
__global__ void __launch_bounds__(kAccThreads) probs_kernel(ProbsArgs a) {
  __shared__ AccShared sh;
  const half* l = a.logits + static_cast<size_t>(blockIdx.x) * a.ld;
  float* out = a.probs + static_cast<size_t>(blockIdx.x) * a.ldp;
  const int n = a.vocab;
  float mx = kNegInf;
  for (int j = threadIdx.x; j < n; j += kAccThreads) mx = fmaxf(mx, __half2float(l[j]));
  mx = block_max(mx, sh);
  for (int j = threadIdx.x; j < n; j += kAccThreads) out[j] = rexp(fdiv(fsub(__half2float(l[j]), mx), a.t));
  __syncthreads();
  RowVec rv;
  rv.p = out;
  float total = chunk_total(rv, n, sh);
  for (int j = threadIdx.x; j < n; j += kAccThreads) out[j] = fdiv(out[j], total);
  __syncthreads();
  if (a.min_p > 0.f && a.min_p < 1.f) {
    float pm = 0.f;
    for (int j = threadIdx.x; j < n; j += kAccThreads) pm = fmaxf(pm, out[j]);
    pm = block_max(pm, sh);
    const float thr = fmul(a.min_p, pm);
    for (int j = threadIdx.x; j < n; j += kAccThreads)
      if (!(out[j] >= thr)) out[j] = 0.f;
    __syncthreads();
    total = chunk_total(rv, n, sh);
    for (int j = threadIdx.x; j < n; j += kAccThreads) out[j] = fdiv(out[j], total);
  }
}

// One draw from a probability row (a draft candidate): out[0] = index.
__global__ void __launch_bounds__(kAccThreads) draw_kernel(DrawArgs a) {
  __shared__ AccShared sh;
  if (threadIdx.x == 0) sh.cursor = a.cursor ? *a.cursor : 0;
  __syncthreads();
  RowVec rv;
  rv.p = a.probs;
  const int pick = walk_row(rv, a.vocab, a.u[sh.cursor + a.u_offset], sh);
  if (threadIdx.x == 0) *a.out = pick >= 0 ? pick : 0;   // a row without a positive entry (non-finite logits)
}

// Acceptance of k candidates against k + 1 target rows.
__global__ void __launch_bounds__(kAccThreads) accept_kernel(AcceptArgs a) {
  __shared__ AccShared sh;
  if (threadIdx.x == 0) sh.cursor = a.cursor ? *a.cursor : 0;
  __syncthreads();
  const double* u = a.u + sh.cursor + a.u_offset;   // k accept draws, then the resample draw
  if (threadIdx.x < kWarp) {
    const int i = threadIdx.x;
    bool ok = false;
    if (i < a.k) {
      const int x = a.cand[i];
      ok = x >= 0 && x < a.vocab &&   // a candidate outside the row is rejected
           fmul(__double2float_rn(u[i]), a.q[static_cast<size_t>(i) * a.ldq + x]) <
           a.p[static_cast<size_t>(i) * a.ldp + x];
    }
    const unsigned rejected = __ballot_sync(0xffffffffu, !ok) & ((a.k < 32 ? (1u << a.k) : 0u) - 1u);
    if (i == 0) sh.n_acc = rejected ? __ffs(rejected) - 1 : a.k;
  }
  __syncthreads();
  const int n = sh.n_acc;
  RowVec rv;
  rv.p = a.p + static_cast<size_t>(n) * a.ldp;
  if (n < a.k) {
    rv.q = a.q + static_cast<size_t>(n) * a.ldq;
    int any = -1;
    for (int j = threadIdx.x; j < a.vocab; j += kAccThreads)
      if (rv(j) > 0.f) any = j;
    if (block_max_int(any, sh) < 0) rv.q = nullptr;   // no positive residual: the target row itself
  }
  const int drawn = walk_row(rv, a.vocab, u[a.k], sh);
  const int tok = drawn >= 0 ? drawn : 0;   // a row without a positive entry (non-finite logits)
  if (threadIdx.x != 0) return;
  if (a.tokens) {
    for (int j = 0; j < n; ++j) a.tokens[j] = a.cand[j];
    a.tokens[n] = tok;
  }
  if (a.n_acc) *a.n_acc = n;
  if (a.state) {
    // the speculative step's bookkeeping (as the greedy accept kernel does)
    int* st = a.state;
    const int base = st[2];
    for (int j = 0; j < n; ++j)
      if (base + j < a.cap_tokens) a.ring[base + j] = a.cand[j];
    if (base + n < a.cap_tokens) a.ring[base + n] = tok;
    st[2] = base + n + 1;
    if (st[3] < a.cap_steps) a.ring_acc[st[3]] = n;
    st[3] += 1;
    st[5] = n == 0 ? st[0] : a.cand[n - 1];
    st[0] = tok;
    st[1] += n + 1;
    st[4] += a.cursor_advance;
  }
}

}  // namespace

cudaError_t launch_probs(const ProbsArgs& a, int rows, cudaStream_t st) {
  if (a.vocab < 1 || a.vocab > kAccMaxChunks * kChunk || rows < 1) return cudaErrorInvalidValue;
  probs_kernel<<<rows, kAccThreads, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_draw(const DrawArgs& a, cudaStream_t st) {
  if (a.vocab < 1 || a.vocab > kAccMaxChunks * kChunk) return cudaErrorInvalidValue;
  draw_kernel<<<1, kAccThreads, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_accept(const AcceptArgs& a, cudaStream_t st) {
  if (a.vocab < 1 || a.vocab > kAccMaxChunks * kChunk || a.k < 1 || a.k > 31) return cudaErrorInvalidValue;
  accept_kernel<<<1, kAccThreads, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace alm
