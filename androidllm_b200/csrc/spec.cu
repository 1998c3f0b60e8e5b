// Device-side bookkeeping of the greedy speculative step
// (androidllm/engine.py:288-320), so a whole step — K draft forwards, one
// (K+1)-row verify forward and the acceptance — runs without the host.
//
// state[0] = token at the current position, state[1] = that position,
// state[2] = tokens emitted in this run, state[3] = steps in this run,
// state[4] = next unused uniform draw (sampling at temperature > 0),
// state[5] = token at position state[1] - 1 (the draft refresh reads it).
#include "common.cuh"
#include "kernels.cuh"

namespace alm {
namespace {

// Inputs of draft forward i: token = (i == 0 ? state token : candidate i-1),
// position = state pos + i.  Also records candidate i-1 from the draft's
// previous pick (row prev_row of its argmax).  With refresh, forward 0 has
// two rows: the token at pos - 1 again, then the state token (the draft
// never forwarded the last candidate of a step that accepted all of them).
__global__ void spec_prep_draft_kernel(const int* state, int* cand, const int* d_argmax, int i,
                                       int* tokens, int* pos, int prev_row, int refresh) {
  if (threadIdx.x != 0) return;
  if (i > 0) {
    cand[i - 1] = d_argmax[prev_row];
    tokens[0] = d_argmax[prev_row];
    pos[0] = state[1] + i;
  } else if (refresh) {
    tokens[0] = state[5];
    tokens[1] = state[0];
    pos[0] = state[1] - 1;
  } else {
    tokens[0] = state[0];
    pos[0] = state[1];
  }
}

// Inputs of the verify forward: [token, c_1 .. c_K] at state pos.
__global__ void spec_prep_verify_kernel(const int* state, int* cand, const int* d_argmax, int k,
                                        int* tokens, int* pos, int prev_row) {
  if (threadIdx.x != 0) return;
  cand[k - 1] = d_argmax[prev_row];
  tokens[0] = state[0];
  for (int j = 0; j < k; ++j) tokens[j + 1] = cand[j];
  pos[0] = state[1];
}

// engine.py:306-320: accept while target pick == candidate; emit the
// accepted candidates and then the target's pick at the first mismatch (or
// the bonus pick after K accepts).
// With sampling, t_argmax holds the target's sampled tokens and the
// candidates are the draft's samples (engine.py:296-320 at T > 0): the step
// consumed k draft draws and n + 1 target draws, so the cursor advances by
// k + n + 1 (the later rows' draws were not used).
__global__ void spec_accept_greedy_kernel(int* state, const int* cand, const int* t_argmax, int k,
                                          int* out_tokens, int* out_accepted, int cap_tokens,
                                          int cap_steps, int sampled) {
  if (threadIdx.x != 0) return;
  int n = 0;
  while (n < k && t_argmax[n] == cand[n]) ++n;
  if (sampled) state[4] += k + n + 1;
  const int base = state[2];
  for (int j = 0; j < n; ++j)
    if (base + j < cap_tokens) out_tokens[base + j] = cand[j];
  if (base + n < cap_tokens) out_tokens[base + n] = t_argmax[n];
  state[2] = base + n + 1;
  if (state[3] < cap_steps) out_accepted[state[3]] = n;
  state[3] += 1;
  state[5] = n == 0 ? state[0] : cand[n - 1];
  state[0] = t_argmax[n];
  state[1] += n + 1;
}

}  // namespace

cudaError_t launch_spec_prep_draft(const int* state, int* cand, const int* d_argmax, int i, int* tokens,
                                   int* pos, int prev_row, int refresh, cudaStream_t st) {
  spec_prep_draft_kernel<<<1, 32, 0, st>>>(state, cand, d_argmax, i, tokens, pos, prev_row, refresh);
  return cudaGetLastError();
}
cudaError_t launch_spec_prep_verify(const int* state, int* cand, const int* d_argmax, int k, int* tokens,
                                    int* pos, int prev_row, cudaStream_t st) {
  spec_prep_verify_kernel<<<1, 32, 0, st>>>(state, cand, d_argmax, k, tokens, pos, prev_row);
  return cudaGetLastError();
}
cudaError_t launch_spec_accept_greedy(int* state, const int* cand, const int* t_argmax, int k, int* out_tokens,
                                      int* out_accepted, int cap_tokens, int cap_steps, int sampled, cudaStream_t st) {
  spec_accept_greedy_kernel<<<1, 32, 0, st>>>(state, cand, t_argmax, k, out_tokens, out_accepted, cap_tokens,
                                              cap_steps, sampled);
  return cudaGetLastError();
}

}  // namespace alm
