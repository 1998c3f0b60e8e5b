// Device sampler: androidllm/engine.py:26-45 (softmax of logits / T, min-p
// keep and renormalise, top-p nucleus in descending-probability order,
// inverse CDF on one uniform draw).  One thread-block cluster of
// kSampleCtas CTAs per row: CTA c holds the row's c-th contiguous slice of
// ceil(V / kSampleCtas) probabilities in shared memory, and the cluster
// combines sums, maxima and radix histograms through distributed shared
// memory.
//
// The arithmetic is fixed so the oracle can restate it bit for bit:
//   * exp is rexp (Cody-Waite reduction + degree-7 Taylor polynomial, every
//     step one correctly rounded fp32 operation, then an exact 2^k scaling);
//   * a row sum: in each slice thread t adds elements t, t + 1024, ... in
//     order, lanes of a warp are added in lane order, warp totals in warp
//     order, and the slice totals in slice order;
//   * probability masses are fixed point, floor(p * 2^52), so the nucleus and
//     the CDF walk are exact integer arithmetic: radix selects (4 rounds of 8
//     bits over the fp32 probability bits) find the element where the
//     descending cumulative mass crosses a target, and ties are resolved by
//     ascending index.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.cuh"

namespace alm {
namespace {

namespace cg = cooperative_groups;

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / kWarp;
constexpr int kSampleCtas = 8;      // cluster size: slices of a row
constexpr int kBuckets = 256;
constexpr int kHistCopies = 16;     // private histogram copies per CTA (2 warps each)
constexpr int kSlots = 8;           // cluster-published values, one slot per reduction
constexpr double kMassScale = 4503599627370496.0;   // 2^52
constexpr int kCountShift = 53;                       // packed histogram word: count << 53 | mass
constexpr unsigned long long kCountOne = 1ull << kCountShift;
constexpr unsigned long long kMassMask = kCountOne - 1;

ALM_DEV float bits_f(uint32_t u) { return __uint_as_float(u); }

// floor(p * 2^52) for 0 <= p <= 1, from the fp32 bits (exact: a shift of the
// 24-bit significand).
ALM_DEV unsigned long long mass_of(float p) {
  const unsigned b = __float_as_uint(p);
  const int e = static_cast<int>(b >> 23);       // biased exponent (sign is 0)
  if (e == 0) return 0;                          // subnormal: p * 2^52 < 2^-45
  const unsigned long long f = (b & 0x7fffffu) | 0x800000u;
  const int sh = e - 127 - 23 + 52;              // p * 2^52 = f * 2^sh
  return sh >= 0 ? f << sh : (sh > -64 ? f >> -sh : 0ull);
}

struct SampleShared {
  float f[kSampleThreads];
  float w[kSampleWarps];
  unsigned long long u64[kSampleWarps];
  unsigned long long u64b[kSampleWarps];
  float bc_f;
  unsigned long long bc_a;
  unsigned long long bc_c;
  int bc_i;
  // published to the cluster (one slot per reduction, never reused)
  float pubf[kSlots];
  unsigned long long pubu[kSlots];
  int pubi[kSlots];
  // this CTA's radix histogram, double-buffered by round parity
  unsigned long long hmass[2][kBuckets];
  unsigned hcnt[2][kBuckets];
  // the cluster's combined histogram of the current round
  unsigned long long tm[kBuckets];
  unsigned long long tc[kBuckets];
};

ALM_DEV float block_max(float v, SampleShared& sh) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) sh.w[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = sh.w[0];
    for (int i = 1; i < kSampleWarps; ++i) m = fmaxf(m, sh.w[i]);
    sh.bc_f = m;
  }
  __syncthreads();
  const float r = sh.bc_f;
  __syncthreads();
  return r;
}

// Fixed-order fp32 total of the per-thread partial sums of this CTA's slice.
ALM_DEV float block_total(float v, SampleShared& sh) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  sh.f[threadIdx.x] = v;
  __syncthreads();
  if (lane == 0) {
    float s = 0.f;
    for (int l = 0; l < kWarp; ++l) s = fadd(s, sh.f[warp * kWarp + l]);
    sh.w[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < kSampleWarps; ++i) s = fadd(s, sh.w[i]);
    sh.bc_f = s;
  }
  __syncthreads();
  const float r = sh.bc_f;
  __syncthreads();
  return r;
}

// Exclusive prefix of per-thread uint64 values over the CTA (exact).
ALM_DEV unsigned long long block_excl_scan(unsigned long long v, SampleShared& sh) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  unsigned long long x = v;
#pragma unroll
  for (int o = 1; o < kWarp; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == kWarp - 1) sh.u64[warp] = x;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long s = 0;
    for (int i = 0; i < kSampleWarps; ++i) {
      const unsigned long long t = sh.u64[i];
      sh.u64[i] = s;
      s += t;
    }
  }
  __syncthreads();
  const unsigned long long r = sh.u64[warp] + x - v;
  __syncthreads();
  return r;
}

// Cluster-wide reductions of one value per CTA through a publication slot.
struct Cluster {
  cg::cluster_group cl;
  int rank;
  SampleShared& sh;

  ALM_DEV float max_f(float v, int slot) {
    if (threadIdx.x == 0) sh.pubf[slot] = v;
    cl.sync();
    float m = kNegInf;
    for (int r = 0; r < kSampleCtas; ++r) m = fmaxf(m, cl.map_shared_rank(sh.pubf, r)[slot]);
    return m;
  }
  // fp32 sum of the CTAs' values in rank order
  ALM_DEV float sum_f(float v, int slot) {
    if (threadIdx.x == 0) sh.pubf[slot] = v;
    cl.sync();
    float s = 0.f;
    for (int r = 0; r < kSampleCtas; ++r) s = fadd(s, cl.map_shared_rank(sh.pubf, r)[slot]);
    return s;
  }
  // exact uint64: total and the sum over lower ranks
  ALM_DEV unsigned long long sum_u(unsigned long long v, int slot, unsigned long long* before) {
    if (threadIdx.x == 0) sh.pubu[slot] = v;
    cl.sync();
    unsigned long long s = 0, b = 0;
    for (int r = 0; r < kSampleCtas; ++r) {
      const unsigned long long x = cl.map_shared_rank(sh.pubu, r)[slot];
      if (r < rank) b += x;
      s += x;
    }
    *before = b;
    return s;
  }
  ALM_DEV int min_i(int v, int slot) {
    if (threadIdx.x == 0) sh.pubi[slot] = v;
    cl.sync();
    int m = 0x7fffffff;
    for (int r = 0; r < kSampleCtas; ++r) m = min(m, cl.map_shared_rank(sh.pubi, r)[slot]);
    return m;
  }
};

struct Crossing {
  unsigned key;                 // fp32 bits of the crossing element's probability
  unsigned long long above;     // mass of all elements with a larger key
  unsigned long long cnt_above; // their count
  bool all_fit;                 // the whole mass is <= target
};

// The element where the descending cumulative mass of the row first exceeds
// `target`: its key and the mass / count of everything before its key.
// `round` counts the radix rounds run so far (histogram buffer parity).
ALM_DEV Crossing find_crossing(const float* p, int n, unsigned long long target, Cluster& c, int& round,
                               unsigned long long* cm) {
  SampleShared& sh = c.sh;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  Crossing x;
  x.above = 0;
  x.cnt_above = 0;
  x.all_fit = false;
  unsigned prefix = 0, mask = 0;
  for (int r = 3; r >= 0; --r, ++round) {
    const int shift = 8 * r, par = round & 1;
    for (int i = threadIdx.x; i < kHistCopies * kBuckets; i += kSampleThreads) cm[i] = 0;
    __syncthreads();
    {
      // one atomic per element: the mass (<= 2^52 per bucket) in the low 53
      // bits, the count (<= 2 warps * ceil(slice / 1024) < 2^11) above
      unsigned long long* m = cm + (warp / (kSampleWarps / kHistCopies)) * kBuckets;
      for (int i = threadIdx.x; i < n; i += kSampleThreads) {
        const float v = p[i];
        const unsigned b = __float_as_uint(v);
        if ((b & mask) == prefix) atomicAdd(&m[(b >> shift) & 0xff], mass_of(v) | kCountOne);
      }
    }
    __syncthreads();
    if (threadIdx.x < kBuckets) {
      unsigned long long m = 0;
      unsigned k = 0;
      for (int h = 0; h < kHistCopies; ++h) {
        const unsigned long long x = cm[h * kBuckets + threadIdx.x];
        m += x & kMassMask;
        k += static_cast<unsigned>(x >> kCountShift);
      }
      sh.hmass[par][threadIdx.x] = m;
      sh.hcnt[par][threadIdx.x] = k;
    }
    c.cl.sync();
    // bucket d's cluster totals; thread j = 255 - d so an inclusive scan over
    // j gives the suffix sums over buckets >= d
    unsigned long long sm = 0, sc = 0;
    if (threadIdx.x < kBuckets) {
      const int d = kBuckets - 1 - threadIdx.x;
      for (int q = 0; q < kSampleCtas; ++q) {
        sm += c.cl.map_shared_rank(&sh.hmass[par][0], q)[d];
        sc += c.cl.map_shared_rank(&sh.hcnt[par][0], q)[d];
      }
      unsigned long long xm = sm, xc = sc;
#pragma unroll
      for (int o = 1; o < kWarp; o <<= 1) {
        const unsigned long long ym = __shfl_up_sync(0xffffffffu, xm, o);
        const unsigned long long yc = __shfl_up_sync(0xffffffffu, xc, o);
        if (lane >= o) {
          xm += ym;
          xc += yc;
        }
      }
      if (lane == kWarp - 1) {
        sh.u64[warp] = xm;
        sh.u64b[warp] = xc;
      }
      sm = xm;   // inclusive within the warp
      sc = xc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      sh.bc_i = -1;
      unsigned long long am = 0, ac = 0;
      for (int w = 0; w < kBuckets / kWarp; ++w) {
        const unsigned long long tm = sh.u64[w], tc = sh.u64b[w];
        sh.u64[w] = am;
        sh.u64b[w] = ac;
        am += tm;
        ac += tc;
      }
    }
    __syncthreads();
    if (threadIdx.x < kBuckets) {
      const int d = kBuckets - 1 - threadIdx.x;
      const unsigned long long suf = x.above + sh.u64[warp] + sm;          // mass of buckets >= d
      const unsigned long long sufc = x.cnt_above + sh.u64b[warp] + sc;
      sh.tm[d] = suf;
      sh.tc[d] = sufc;
    }
    __syncthreads();
    if (threadIdx.x < kBuckets) {
      const int d = threadIdx.x;
      const unsigned long long suf = sh.tm[d];
      const unsigned long long above_d = d + 1 < kBuckets ? sh.tm[d + 1] : x.above;   // mass of buckets > d
      if (suf > target && above_d <= target) {
        sh.bc_i = d;
        sh.bc_a = above_d;
        sh.bc_c = d + 1 < kBuckets ? sh.tc[d + 1] : x.cnt_above;
      }
    }
    __syncthreads();
    const int sel = sh.bc_i;
    if (sel >= 0) {
      x.above = sh.bc_a;
      x.cnt_above = sh.bc_c;
    }
    __syncthreads();
    if (sel < 0) {
      x.all_fit = true;
      x.key = 0;
      return x;
    }
    prefix |= static_cast<unsigned>(sel) << shift;
    mask |= 0xffu << shift;
  }
  x.key = prefix;
  return x;
}

// The j-th element (0-based, ascending row index) whose key equals `key`:
// the CTA that holds it writes lo + its slice index into *out.
ALM_DEV void jth_with_key(const float* p, int n, int lo, unsigned key, unsigned long long j, Cluster& c,
                          int slot, int* out) {
  const int seg = (n + kSampleThreads - 1) / kSampleThreads;
  const int a = min(n, static_cast<int>(threadIdx.x) * seg), b = min(n, a + seg);
  unsigned long long k = 0;
  for (int i = a; i < b; ++i) k += __float_as_uint(p[i]) == key;
  const unsigned long long in_cta = block_excl_scan(k, c.sh);
  unsigned long long cta_k = in_cta + k;   // running count; the last thread holds the CTA total
  if (threadIdx.x == kSampleThreads - 1) c.sh.bc_a = cta_k;
  __syncthreads();
  cta_k = c.sh.bc_a;
  __syncthreads();
  unsigned long long before;
  c.sum_u(cta_k, slot, &before);
  const unsigned long long first = before + in_cta;
  if (j >= first && j < first + k) {
    unsigned long long q = first;
    for (int i = a; i < b; ++i)
      if (__float_as_uint(p[i]) == key) {
        if (q == j) {
          *out = lo + i;
          break;
        }
        ++q;
      }
  }
}

// First row index whose inclusive cumulative mass (index order) exceeds
// `target`; the CTA that holds it writes it into *out.
ALM_DEV void first_cum_above(const float* p, int n, int lo, unsigned long long target, Cluster& c, int slot,
                             int* out) {
  const int seg = (n + kSampleThreads - 1) / kSampleThreads;
  const int a = min(n, static_cast<int>(threadIdx.x) * seg), b = min(n, a + seg);
  unsigned long long m = 0;
  for (int i = a; i < b; ++i) m += mass_of(p[i]);
  const unsigned long long in_cta = block_excl_scan(m, c.sh);
  if (threadIdx.x == kSampleThreads - 1) c.sh.bc_a = in_cta + m;
  __syncthreads();
  const unsigned long long cta_m = c.sh.bc_a;
  __syncthreads();
  unsigned long long before;
  c.sum_u(cta_m, slot, &before);
  const unsigned long long start = before + in_cta;
  if (target >= start && target < start + m) {
    unsigned long long q = start;
    for (int i = a; i < b; ++i) {
      q += mass_of(p[i]);
      if (q > target) {
        *out = lo + i;
        break;
      }
    }
  }
}

__global__ void __launch_bounds__(kSampleThreads, 1) sample_kernel(SampleArgs a, int slice) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ SampleShared sh;
  float* p = reinterpret_cast<float*>(smem);
  unsigned long long* cm = reinterpret_cast<unsigned long long*>(smem + ((static_cast<size_t>(slice) * 4 + 15) & ~15));
  Cluster c{cg::this_cluster(), 0, sh};
  c.rank = static_cast<int>(c.cl.block_rank());
  grid_dep_wait();
  const int row = blockIdx.y, V = a.vocab;
  const int lo = min(V, c.rank * slice), hi = min(V, lo + slice), n = hi - lo;
  const half* lg = a.logits + static_cast<size_t>(row) * a.ld;
  int* out = a.out + row;
  const int ubase = a.u_cursor ? *a.u_cursor : 0;
  const double u = a.uniforms ? a.uniforms[ubase + a.u_offset + row] : 0.0;

  // the slice's logits (16-byte loads when aligned), the row maximum
  float mx = kNegInf;
  const half* src = lg + lo;
  if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const int n8 = n / 8;
    for (int base = 0; base < n8; base += kSampleThreads * 4) {
      uint4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = base + j * kSampleThreads + static_cast<int>(threadIdx.x);
        v[j] = i < n8 ? __ldg(reinterpret_cast<const uint4*>(src) + i) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = base + j * kSampleThreads + static_cast<int>(threadIdx.x);
        if (i < n8) {
          const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float f = __half2float(__ushort_as_half(static_cast<unsigned short>(
                (e & 1) ? (w[e >> 1] >> 16) : (w[e >> 1] & 0xffffu))));
            p[i * 8 + e] = f;
            mx = fmaxf(mx, f);
          }
        }
      }
    }
    for (int i = n8 * 8 + static_cast<int>(threadIdx.x); i < n; i += kSampleThreads) {
      const float f = __half2float(src[i]);
      p[i] = f;
      mx = fmaxf(mx, f);
    }
  } else {
    for (int i = threadIdx.x; i < n; i += kSampleThreads) {
      const float v = __half2float(src[i]);
      p[i] = v;
      mx = fmaxf(mx, v);
    }
  }
  mx = c.max_f(block_max(mx, sh), 0);

  if (!(a.temperature > 0.f)) {   // T <= 0: argmax, first index of the maximum
    int first = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += kSampleThreads)
      if (p[i] == mx) {
        first = lo + i;
        break;
      }
    first = -static_cast<int>(block_max(-static_cast<float>(first == 0x7fffffff ? V : first), sh));
    first = c.min_i(first, 0);
    if (c.rank == 0 && threadIdx.x == 0) *out = first;
  } else {
    // softmax(l / T): rexp, fixed-order total
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += kSampleThreads) {
      const float e = rexp(fdiv(fsub(p[i], mx), a.temperature));
      p[i] = e;
      s = fadd(s, e);
    }
    const float total = c.sum_f(block_total(s, sh), 1);
    // min-p: keep p >= min_p * max(p) (max(p) = 1 / total: the top element's exp is 1), renormalise
    const bool use_min_p = a.min_p > 0.f && a.min_p < 1.f;
    const float thr = use_min_p ? fmul(a.min_p, fdiv(1.f, total)) : 0.f;
    float total2 = 1.f;
    if (use_min_p) {
      float s2 = 0.f;
      for (int i = threadIdx.x; i < n; i += kSampleThreads) {
        const float q = fdiv(p[i], total);
        s2 = fadd(s2, q >= thr ? q : 0.f);
      }
      total2 = c.sum_f(block_total(s2, sh), 2);
    }
    for (int i = threadIdx.x; i < n; i += kSampleThreads) {
      float q = fdiv(p[i], total);
      if (use_min_p) q = q >= thr ? fdiv(q, total2) : 0.f;
      p[i] = q;
    }
    __syncthreads();

    int round = 0;
    if (a.top_p < 1.f) {
      // nucleus: the descending prefix with cumulative mass <= floor(top_p * 2^52)
      const unsigned long long budget = __double2ull_rz(static_cast<double>(a.top_p) * kMassScale);
      const Crossing c1 = find_crossing(p, n, budget, c, round, cm);
      unsigned long long n_mass, n_keep;
      if (c1.all_fit) {
        unsigned long long m = 0, before;
        for (int i = threadIdx.x; i < n; i += kSampleThreads) m += mass_of(p[i]);
        const unsigned long long cta_m = block_excl_scan(m, sh) + m;
        if (threadIdx.x == kSampleThreads - 1) sh.bc_a = cta_m;
        __syncthreads();
        n_mass = c.sum_u(sh.bc_a, 3, &before);
        n_keep = V;
      } else {
        const unsigned long long mk = mass_of(__uint_as_float(c1.key));
        const unsigned long long j1 = (budget - c1.above) / mk;
        n_keep = c1.cnt_above + j1;
        n_mass = c1.above + j1 * mk;
      }
      if (n_keep == 0) {
        // only the top element: the largest probability, lowest index
        float pm = kNegInf;
        for (int i = threadIdx.x; i < n; i += kSampleThreads) pm = fmaxf(pm, p[i]);
        pm = c.max_f(block_max(pm, sh), 4);
        jth_with_key(p, n, lo, __float_as_uint(pm), 0, c, 5, out);
      } else {
        unsigned long long target = __double2ull_rz(u * static_cast<double>(n_mass));
        if (target >= n_mass) target = n_mass - 1;
        const Crossing c2 = find_crossing(p, n, target, c, round, cm);
        const unsigned long long mk = mass_of(__uint_as_float(c2.key));
        jth_with_key(p, n, lo, c2.key, (target - c2.above) / mk, c, 5, out);
      }
    } else {
      unsigned long long m = 0, before;
      for (int i = threadIdx.x; i < n; i += kSampleThreads) m += mass_of(p[i]);
      const unsigned long long cta_m = block_excl_scan(m, sh) + m;
      if (threadIdx.x == kSampleThreads - 1) sh.bc_a = cta_m;
      __syncthreads();
      const unsigned long long tot = c.sum_u(sh.bc_a, 3, &before);
      unsigned long long target = __double2ull_rz(u * static_cast<double>(tot));
      if (target >= tot) target = tot - 1;
      first_cum_above(p, n, lo, target, c, 6, out);
    }
  }
  grid_dep_launch();
  c.cl.sync();   // peers may still read this CTA's shared memory
}

}  // namespace

size_t sample_smem_bytes(int vocab) {
  const size_t slice = (static_cast<size_t>(vocab) + kSampleCtas - 1) / kSampleCtas;
  return ((slice * 4 + 15) & ~static_cast<size_t>(15)) + static_cast<size_t>(kHistCopies) * kBuckets * sizeof(unsigned long long);
}

constexpr size_t kSampleMaxSmem = 200 * 1024;

cudaError_t sample_init_attrs() {
  return cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kSampleMaxSmem));
}

cudaError_t launch_sample(const SampleArgs& a, int rows, bool pdl, cudaStream_t st) {
  if (rows < 1 || a.vocab < 1) return cudaErrorInvalidValue;
  const size_t smem = sample_smem_bytes(a.vocab);
  if (smem > kSampleMaxSmem) return cudaErrorInvalidValue;
  const int slice = (a.vocab + kSampleCtas - 1) / kSampleCtas;
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(kSampleCtas, rows);
  c.blockDim = dim3(kSampleThreads);
  c.dynamicSmemBytes = smem;
  c.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kSampleCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  c.attrs = attr;
  c.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&c, sample_kernel, a, slice);
}

}  // namespace alm
