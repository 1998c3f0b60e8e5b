// Interface of the cluster forward kernel (cluster_fwd.cu): every layer of a
// single-row forward in one launch of one 16-CTA thread-block cluster.
#pragma once
#include "forward.cuh"

namespace alm {

constexpr int kCfCtas = 16;          // CTAs of the cluster (non-portable size)
constexpr int kCfSlots = 14;         // weight ring slots per CTA
constexpr int kCfSlotBytes = 8192;   // bytes per slot (whole records)
constexpr int kCfMaxItems = 128;     // (tile, k-range) items per CTA and GEMV

// The share of one GEMV a cluster CTA streams and decodes: output tiles
// [t0, t1) with all their k-blocks (one contiguous run of records), split into
// items of (tile, one of the S = ksw * ksg K splits of kps k-blocks of the
// standalone launch shape), streamed in chunks of R records.
struct CfPlan {
  int t0 = 0, t1 = 0, S = 1, kps = 1, R = 1, n_items = 0, n_rec = 0, n_chunks = 0;
  int rec_bytes = 0;
  const unsigned char* base = nullptr;
};
__host__ __device__ CfPlan cluster_fwd_plan(const QTile& w, int cta);
// The weight can run in the cluster kernel (tile layout, shape limits).
bool cluster_fwd_weight_ok(const QTile& w);
// Dynamic shared memory of the kernel for a model whose widest GEMV input
// has max_k_blocks 64-column blocks.
size_t cluster_fwd_smem_bytes(int max_k_blocks, int head_dim);
// Sets the kernel's attributes on the current device; *n_clusters = clusters
// that fit on the device at once (0: the kernel cannot run here).
cudaError_t cluster_fwd_init(size_t smem_bytes, int* n_clusters);
// Embedding and every layer for one row (p.M must be 1); the caller runs the
// final norm and the head.
cudaError_t launch_cluster_fwd(const FwdParams& p, size_t smem_bytes, bool pdl, cudaStream_t st);

}  // namespace alm
