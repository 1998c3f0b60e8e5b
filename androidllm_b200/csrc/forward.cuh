// Interface of the persistent forward kernel (forward.cu).
#pragma once
#include "kernels.cuh"

namespace alm {

// Barrier arrivals reserved per launch (per CTA); a forward needs
// forward_barriers() of them.
constexpr int kBarRound = 4096;
// Rows (verify tokens) a persistent forward takes: one n8 MMA tile.
constexpr int kPersistRows = 8;

// Device copy of one layer's weights and norms.
struct FwdLayer {
  QTile qkv, o, gu, down;
  const half* n_in = nullptr;
  const half* n_post = nullptr;
};

struct FwdParams {
  const FwdLayer* layers = nullptr;
  int n_layers = 0;
  int M = 1;                    // activation rows (1..8)
  int hidden = 0, inter = 0, heads = 0, kv_heads = 0, head_dim = 0, vocab = 0;
  float eps = 0.f;
  float sqrt_hd = 1.f;          // attention score divisor
  EmbedArgs embed;              // tokens -> embed.out (layer 0 input)
  // workspace
  half* s1 = nullptr;
  half* s2 = nullptr;
  float* ss1 = nullptr;
  float* ss2 = nullptr;
  float* q = nullptr;
  half* ctx = nullptr;
  half* h = nullptr;
  half* xn = nullptr;
  half* logits = nullptr;
  float* part = nullptr;
  // paged KV cache and attention scratch
  half* kcache = nullptr;
  half* vcache = nullptr;
  size_t kv_layer_elems = 0;
  const int* page_table = nullptr;
  int page_size = 16;
  int max_ctx = 0;
  float* scores = nullptr;
  int score_ld = 0;
  float* stats = nullptr;
  const half* rope = nullptr;
  // final norm, head, argmax
  int do_head = 1;
  QTile head;
  const half* final_norm = nullptr;
  float* am_val = nullptr;
  int* am_idx = nullptr;
  int* argmax = nullptr;
  StepIO io;
  unsigned long long* bar = nullptr;   // grid-barrier arrival counter
  // Optional phase trace (global timer, ns): arrival time of every CTA at
  // every barrier, [barrier][cta], then the time CTA 0 left each barrier.
  unsigned long long* trace = nullptr;
  int trace_cap = 0;   // entries of trace (cluster forward)
};

__host__ __device__ int forward_barriers(int n_layers, bool head);
// Dynamic shared memory of the kernel for the model's largest GEMV staging.
size_t forward_smem_bytes(size_t max_stage_bytes, int head_dim, int hidden);
// Sets the kernel's shared-memory limit; returns the resident CTAs per SM.
cudaError_t forward_init_attrs(size_t smem_bytes, int* ctas_per_sm);
cudaError_t launch_forward(const FwdParams& p, int grid, size_t smem_bytes, cudaStream_t st);

}  // namespace alm
