// Attention of a decode / verify pass in one launch.  Block (chunk c, kv
// head, row group) = the two-pass scheme's scores block, continued:
//   1. the V rows of its 64-position chunk are copied to shared memory
//      (cp.async) while attn_scores_body computes the chunk's scores and
//      statistics exactly as the scores pass does;
//   2. it publishes its statistics (fence + count) and waits until every
//      chunk of its (kv head, row group) has published (bounded: a wait that
//      gives up sets err = 2 and the block carries on);
//   3. it combines the chunk statistics in the P.V pass's fixed order, forms
//      P = fp16(exp(s - max) / sum) for its chunk — the same probabilities,
//      bit for bit, as the two passes — and multiplies them with its V rows
//      on the tensor cores into an fp32 partial (16 rows x head_dim);
//   4. the last block of the (kv head, row group) to finish adds the chunk
//      partials in chunk order, writes the fp16 context rows and resets the
//      count and the ticket.
// Every block of the grid must be resident at once for step 2 to end, so the
// launcher takes the kernel only when the grid fits (occupancy x SMs) and the
// dependent launch is released only at the very end.  Results differ from
// the two passes in the fp32 order of the P.V sums (per chunk, then across
// chunks); every pass that takes this kernel (1-row decode, k+1-row verify,
// multi-sequence) has the same order, so verify rows still equal single rows
// bit for bit.
#include "attn_body.cuh"

namespace alm {
namespace {

constexpr int kFzThreads = kAttnThreads;
constexpr long long kFzSpinLimit = 1ll << 22;   // polls of the count (~0.3 s with the sleeps)

__host__ __device__ inline size_t fz_v_offset(int hd) { return attn_scores_smem(hd); }
__host__ __device__ inline int fz_vld(int hd) { return hd + 8; }
__host__ __device__ inline size_t fz_p_offset(int hd) {
  return fz_v_offset(hd) + static_cast<size_t>(kAttnChunk) * fz_vld(hd) * sizeof(half);
}
constexpr int kFzPld = kAttnChunk + 8;   // P row stride (halves)
__host__ __device__ inline size_t fz_smem(int hd) {
  return fz_p_offset(hd) + static_cast<size_t>(kAttnRows) * kFzPld * sizeof(half);
}

ALM_DEV void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
ALM_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

ALM_DEV unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Row max and sum over a row group's chunk statistics: one warp per row,
// lane l takes chunks l, l + 32, ... in order, then a butterfly — the P.V
// pass's arithmetic (attn_pv_body).
ALM_DEV void fz_row_stats(const float* st, int rl, int n_chunks, int lane, float& mx_out, float& l_out) {
  float mx = kNegInf;
  for (int c = lane; c < n_chunks; c += 32) mx = fmaxf(mx, __ldcg(st + (c * kAttnRows + rl) * 2));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float l = 0.f;
  for (int c = lane; c < n_chunks; c += 32) {
    const float m = __ldcg(st + (c * kAttnRows + rl) * 2);
    if (m != kNegInf) l = fadd(l, fmul(__ldcg(st + (c * kAttnRows + rl) * 2 + 1), expf(m - mx)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) l = fadd(l, __shfl_xor_sync(0xffffffffu, l, o));
  mx_out = mx;
  l_out = l;
}

__global__ void __launch_bounds__(kFzThreads) attn_fused_kernel(AttnArgs a, float inv_sqrt_den) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ AttnShared sh;
  __shared__ float s_m[kAttnRows], s_l[kAttnRows];
  __shared__ int s_last;
  const int chunk = blockIdx.x, kvh = blockIdx.y, rg = blockIdx.z;
  attn_scores_pages(a, chunk, smem_raw);   // the page table is not written by earlier kernels
  __syncthreads();
  grid_dep_wait();

  const int hd = a.head_dim, tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const AttnSeqView sv = attn_seq_view(a, rg, false);
  const int n_ctx = sv.pos0 + sv.n_tok;
  const int c0 = chunk * kAttnChunk;
  if (c0 >= n_ctx) return;   // not part of this pass (its context is shorter)
  const int n_chunks = (n_ctx + kAttnChunk - 1) / kAttnChunk;
  const int n_chunks_max = gridDim.x;
  const int gq = a.heads / a.kv_heads;
  const int n_rows = sv.n_tok * gq;
  const int n_rg = attn_row_groups(a);
  const int lg = sv.local;

  // 1. V rows of the chunk -> shared memory (in flight during the scores)
  half* vs = reinterpret_cast<half*>(smem_raw + fz_v_offset(hd));
  const int vld = fz_vld(hd);
  {
    const int* s_pg = attn_scores_pg(a, smem_raw);
    if (a.seqs) {
      // a multi-sequence pass stages its pages in the scores body: read them
      // from the sequence's page table here
      const int vpr = hd / 8;
      for (int i = tid; i < kAttnChunk * vpr; i += kFzThreads) {
        const int p = c0 + i / vpr;
        if (p < n_ctx) {
          const int page = __ldcg(sv.ptab + p / a.page_size);
          const half* row = a.vcache + ((static_cast<size_t>(page) * a.kv_heads + kvh) * a.page_size +
                                        p % a.page_size) * hd;
          cp_async16(vs + (i / vpr) * vld + (i % vpr) * 8, row + (i % vpr) * 8);
        }
      }
    } else {
      const int pg0 = c0 / a.page_size;
      const int vpr = hd / 8;
      for (int i = tid; i < kAttnChunk * vpr; i += kFzThreads) {
        const int p = c0 + i / vpr;
        if (p < n_ctx)
          cp_async16(vs + (i / vpr) * vld + (i % vpr) * 8,
                     kv_row(a.vcache, s_pg, pg0, a.page_size, a.kv_heads, kvh, hd, p) + (i % vpr) * 8);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }

  // scores and statistics of this chunk (exactly the scores pass)
  attn_scores_body(a, inv_sqrt_den, chunk, kvh, rg, n_chunks_max, smem_raw, sh);

  // 2. publish, then wait for every chunk of this (kv head, row group)
  const size_t key = static_cast<size_t>(kvh) * n_rg + rg;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    atomicAdd(a.fz_count + key, 1u);
    long long spins = 0;
    while (ld_acquire_u32(a.fz_count + key) < static_cast<unsigned>(n_chunks)) {
      if (++spins > kFzSpinLimit) {
        if (a.err) atomicExch(a.err, 2);
        break;
      }
      __nanosleep(64);
    }
    __threadfence();
  }
  __syncthreads();

  // 3. row statistics (fixed order), P of this chunk, P.V partial
  const float* st = a.stats + (key * n_chunks_max) * kAttnRows * 2;
  for (int rl = warp; rl < kAttnRows; rl += kFzThreads / kWarp) {
    float mx, l;
    fz_row_stats(st, rl, n_chunks, lane, mx, l);
    if (lane == 0) {
      s_m[rl] = mx;
      s_l[rl] = l;
    }
  }
  __syncthreads();
  half* ps = reinterpret_cast<half*>(smem_raw + fz_p_offset(hd));
  const size_t srow0 = key * kAttnRows;
  for (int i = tid; i < kAttnRows * kAttnChunk; i += kFzThreads) {
    const int rl = i / kAttnChunk, pc = i % kAttnChunk, p = c0 + pc;
    const int r = lg * kAttnRows + rl;
    float pv = 0.f;
    if (r < n_rows && p < n_ctx) {
      const float s = __ldcg(a.scores + (srow0 + rl) * a.score_ld + p);
      if (s != kNegInf) pv = fdiv(expf(s - s_m[rl]), s_l[rl]);
    }
    ps[rl * kFzPld + pc] = __float2half_rn(pv);
  }
  cp_async_wait_all();
  // rows of V past the context were not copied: zero them (their P is 0,
  // but 0 x NaN would not be)
  for (int i = tid; i < kAttnChunk * (hd / 8); i += kFzThreads) {
    const int pr = i / (hd / 8);
    if (c0 + pr >= n_ctx) *reinterpret_cast<uint4*>(vs + pr * vld + (i % (hd / 8)) * 8) = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();

  const int nds = hd / 16;
  float* part = a.fz_part + (key * n_chunks_max + chunk) * kAttnRows * hd;
  const int g = lane >> 2, t = lane & 3;
  for (int ds = warp; ds < nds; ds += kFzThreads / kWarp) {
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < kAttnChunk / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(a0, a1, a2, a3, ps + (lane % 16) * kFzPld + kk * 16 + (lane / 16) * 8);
      uint32_t b0, b1, b2, b3;
      const int vrow = kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
      ldmatrix_x4_trans(b0, b1, b2, b3, vs + vrow * vld + ds * 16 + (lane / 16) * 8);
      mma16816(acc[0], a0, a1, a2, a3, b0, b1);
      mma16816(acc[1], a0, a1, a2, a3, b2, b3);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rl = g + 8 * (e >> 1), d = ds * 16 + nt * 8 + 2 * t + (e & 1);
        part[rl * hd + d] = acc[nt][e];
      }
  }

  // 4. the last block adds the chunk partials in order
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(a.fz_ticket + key, 1u) == static_cast<unsigned>(n_chunks - 1);
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    const float* base = a.fz_part + key * n_chunks_max * kAttnRows * hd;
    const size_t stride = static_cast<size_t>(kAttnRows) * hd;
    for (int i = tid; i < kAttnRows * hd; i += kFzThreads) {
      const int rl = i / hd, d = i % hd;
      const int r = lg * kAttnRows + rl;
      // loads of 8 chunks in flight at a time, added in chunk order
      float v = 0.f;
      for (int c0b = 0; c0b < n_chunks; c0b += 8) {
        float x[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = c0b + j < n_chunks ? __ldcg(base + (c0b + j) * stride + i) : 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (c0b + j < n_chunks) v = c0b + j == 0 ? x[j] : fadd(v, x[j]);
      }
      if (r < n_rows) {
        const int m = sv.m0 + r / gq, head = kvh * gq + r % gq;
        a.ctx[static_cast<size_t>(m) * a.ldc + head * hd + d] = __float2half_rn(v);
      }
    }
    if (tid == 0) {
      atomicExch(a.fz_count + key, 0u);
      atomicExch(a.fz_ticket + key, 0u);
    }
  }
  grid_dep_launch();
}

int g_fz_capacity = 0;   // blocks of the kernel resident at once on the device

}  // namespace

cudaError_t attn_fused_init_attrs(int n_sms) {
  cudaError_t e = cudaFuncSetAttribute(attn_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(fz_smem(256)));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_fused_kernel, kFzThreads, fz_smem(128));
  if (e != cudaSuccess) return e;
  g_fz_capacity = per_sm * n_sms;
  return cudaSuccess;
}

bool attn_fused_ok(const AttnArgs& a) {
  if (!a.fz_count || !a.fz_ticket || !a.fz_part || a.head_dim % 16 != 0 || a.head_dim > 128) return false;
  const long long blocks = static_cast<long long>(attn_chunks_max(a)) * a.kv_heads * attn_row_groups(a);
  return blocks <= g_fz_capacity;
}

cudaError_t launch_attn_fused(const AttnArgs& a, bool pdl, cudaStream_t st) {
  if (!attn_fused_ok(a)) return cudaErrorInvalidValue;
  const float den = static_cast<float>(sqrt(static_cast<double>(a.head_dim)));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(attn_chunks_max(a), a.kv_heads, attn_row_groups(a));
  c.blockDim = dim3(kFzThreads);
  c.dynamicSmemBytes = fz_smem(a.head_dim);
  c.stream = st;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&c, attn_fused_kernel, a, den);
}

}  // namespace alm
