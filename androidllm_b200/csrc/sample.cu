// Device sampler: androidllm/engine.py:26-45 (softmax of logits / T, min-p
// keep and renormalise, top-p nucleus in descending-probability order,
// inverse CDF on one uniform draw) for one row of logits per CTA.
//
// The arithmetic is fixed so the oracle can restate it bit for bit:
//   * exp is rexp (Cody-Waite reduction + degree-7 Taylor polynomial, every
//     step one correctly rounded fp32 operation, then an exact 2^k scaling);
//   * a block sum: thread t adds elements t, t + 1024, ... in order, lanes of
//     a warp are added in lane order, warp totals in warp order;
//   * probability masses are fixed point, floor(p * 2^52), so the nucleus and
//     the CDF walk are exact integer arithmetic: radix selects (4 rounds of 8
//     bits over the fp32 probability bits, per-warp 64-bit histograms) find
//     the element where the descending cumulative mass crosses a target, and
//     ties are resolved by ascending index.
#include "common.cuh"
#include "kernels.cuh"

namespace alm {
namespace {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / kWarp;
constexpr int kBuckets = 256;
constexpr double kMassScale = 4503599627370496.0;   // 2^52

ALM_DEV float bits_f(uint32_t u) { return __uint_as_float(u); }

// exp(x) for fp32 x <= 0 from correctly rounded fp32 operations only.
ALM_DEV float rexp(float x) {
  const float log2e = bits_f(0x3fb8aa3bu);
  const float ln2_hi = bits_f(0x3f317200u);   // fp32(ln 2) with its low 9 mantissa bits cleared
  const float ln2_lo = bits_f(0x35bfbe8eu);   // fp32(ln 2 - ln2_hi)
  const float k = rintf(fmul(x, log2e));
  const float r = fsub(fsub(x, fmul(k, ln2_hi)), fmul(k, ln2_lo));
  // 1/7!, 1/6!, ..., 1/1!, 1/0! in Horner order
  const uint32_t c[8] = {0x39500d01u, 0x3ab60b61u, 0x3c088889u, 0x3d2aaaabu,
                         0x3e2aaaabu, 0x3f000000u, 0x3f800000u, 0x3f800000u};
  float acc = bits_f(c[0]);
#pragma unroll
  for (int i = 1; i < 8; ++i) acc = fadd(fmul(acc, r), bits_f(c[i]));
  const float out = ldexpf(acc, static_cast<int>(k));
  return x < bits_f(0xc2ae0000u) ? 0.f : out;   // below -87: 0
}

ALM_DEV unsigned long long mass_of(float p) { return __double2ull_rz(static_cast<double>(p) * kMassScale); }

struct SampleShared {
  float f[kSampleThreads];
  float w[kSampleWarps];
  unsigned long long u64[kSampleWarps];
  float bc_f;
  unsigned long long bc_a, bc_b;
  unsigned bc_key, bc_cnt;
  int bc_i, bc_flag;
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

// Fixed-order fp32 total of the per-thread partial sums.
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

// Exclusive prefix of per-thread uint64 values (exact); total in *tot.
ALM_DEV unsigned long long block_excl_scan(unsigned long long v, unsigned long long* tot, SampleShared& sh) {
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
    sh.bc_a = s;
  }
  __syncthreads();
  const unsigned long long r = sh.u64[warp] + x - v;
  *tot = sh.bc_a;
  __syncthreads();
  return r;
}

struct Crossing {
  unsigned key;                 // fp32 bits of the crossing element's probability
  unsigned long long above;     // mass of all elements with a larger key
  unsigned cnt_above;           // their count
  bool all_fit;                 // the whole mass is <= target
};

// The element where the descending cumulative mass first exceeds `target`:
// its key and the mass / count of everything before its key.
ALM_DEV Crossing find_crossing(const float* p, int V, unsigned long long target, SampleShared& sh,
                               unsigned long long* hmass, unsigned* hcnt) {
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  Crossing c;
  c.above = 0;
  c.cnt_above = 0;
  c.all_fit = false;
  unsigned prefix = 0, mask = 0;
  for (int r = 3; r >= 0; --r) {
    const int shift = 8 * r;
    for (int i = threadIdx.x; i < kSampleWarps * kBuckets; i += kSampleThreads) {
      hmass[i] = 0;
      hcnt[i] = 0;
    }
    __syncthreads();
    unsigned long long* wm = hmass + warp * kBuckets;
    unsigned* wc = hcnt + warp * kBuckets;
    for (int i = threadIdx.x; i < V; i += kSampleThreads) {
      const float v = p[i];
      const unsigned k = __float_as_uint(v);
      if ((k & mask) == prefix) {
        const int d = (k >> shift) & 0xff;
        atomicAdd(&wm[d], mass_of(v));
        atomicAdd(&wc[d], 1u);
      }
    }
    __syncthreads();
    // combine the warps' histograms (exact) into warp 0's row
    for (int d = threadIdx.x; d < kBuckets; d += kSampleThreads) {
      unsigned long long m = 0;
      unsigned n = 0;
      for (int w = 0; w < kSampleWarps; ++w) {
        m += hmass[w * kBuckets + d];
        n += hcnt[w * kBuckets + d];
      }
      hmass[d] = m;
      hcnt[d] = n;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int sel = -1;
      unsigned long long above = c.above;
      unsigned cnt = c.cnt_above;
      for (int d = kBuckets - 1; d >= 0; --d) {
        if (above + hmass[d] <= target) {
          above += hmass[d];
          cnt += hcnt[d];
        } else {
          sel = d;
          break;
        }
      }
      sh.bc_i = sel;
      sh.bc_a = above;
      sh.bc_cnt = cnt;
    }
    __syncthreads();
    const int sel = sh.bc_i;
    c.above = sh.bc_a;
    c.cnt_above = sh.bc_cnt;
    __syncthreads();
    if (sel < 0) {
      c.all_fit = true;
      c.key = 0;
      return c;
    }
    prefix |= static_cast<unsigned>(sel) << shift;
    mask |= 0xffu << shift;
  }
  (void)lane;
  c.key = prefix;
  return c;
}

// Index of the j-th element (0-based, ascending index) whose key equals `key`.
ALM_DEV int jth_with_key(const float* p, int V, unsigned key, unsigned long long j, SampleShared& sh) {
  const int seg = (V + kSampleThreads - 1) / kSampleThreads;
  const int lo = min(V, threadIdx.x * seg), hi = min(V, lo + seg);
  unsigned long long n = 0;
  for (int i = lo; i < hi; ++i) n += __float_as_uint(p[i]) == key;
  unsigned long long tot;
  const unsigned long long before = block_excl_scan(n, &tot, sh);
  if (threadIdx.x == 0) sh.bc_i = -1;
  __syncthreads();
  if (j >= before && j < before + n) {
    unsigned long long c = before;
    for (int i = lo; i < hi; ++i)
      if (__float_as_uint(p[i]) == key) {
        if (c == j) {
          sh.bc_i = i;
          break;
        }
        ++c;
      }
  }
  __syncthreads();
  const int r = sh.bc_i;
  __syncthreads();
  return r;
}

// First index whose inclusive cumulative mass (index order) exceeds target.
ALM_DEV int first_cum_above(const float* p, int V, unsigned long long target, SampleShared& sh) {
  const int seg = (V + kSampleThreads - 1) / kSampleThreads;
  const int lo = min(V, threadIdx.x * seg), hi = min(V, lo + seg);
  unsigned long long m = 0;
  for (int i = lo; i < hi; ++i) m += mass_of(p[i]);
  unsigned long long tot;
  const unsigned long long before = block_excl_scan(m, &tot, sh);
  if (threadIdx.x == 0) sh.bc_i = V - 1;
  __syncthreads();
  if (target >= before && target < before + m) {
    unsigned long long c = before;
    for (int i = lo; i < hi; ++i) {
      c += mass_of(p[i]);
      if (c > target) {
        sh.bc_i = i;
        break;
      }
    }
  }
  __syncthreads();
  const int r = sh.bc_i;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kSampleThreads, 1) sample_kernel(SampleArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ SampleShared sh;
  unsigned long long* hmass = reinterpret_cast<unsigned long long*>(smem);          // [warps][256]
  unsigned* hcnt = reinterpret_cast<unsigned*>(hmass + kSampleWarps * kBuckets);     // [warps][256]
  grid_dep_wait();
  const int row = blockIdx.x, V = a.vocab;
  const half* lg = a.logits + static_cast<size_t>(row) * a.ld;
  float* p = a.scratch + static_cast<size_t>(row) * V;
  const int ubase = a.u_cursor ? *a.u_cursor : 0;
  const double u = a.uniforms[ubase + a.u_offset + row];

  // softmax(l / T): max, rexp, fixed-order total
  float mx = kNegInf;
  for (int i = threadIdx.x; i < V; i += kSampleThreads) mx = fmaxf(mx, __half2float(lg[i]));
  mx = block_max(mx, sh);
  if (!(a.temperature > 0.f)) {   // T <= 0: argmax, first index of the maximum
    int first = V;
    for (int i = threadIdx.x; i < V; i += kSampleThreads)
      if (__half2float(lg[i]) == mx) {
        first = i;
        break;
      }
    first = -static_cast<int>(block_max(static_cast<float>(-first), sh));
    if (threadIdx.x == 0) a.out[row] = first;
    return;
  }
  float s = 0.f;
  for (int i = threadIdx.x; i < V; i += kSampleThreads) {
    const float e = rexp(fdiv(fsub(__half2float(lg[i]), mx), a.temperature));
    p[i] = e;
    s = fadd(s, e);
  }
  const float total = block_total(s, sh);
  // min-p: keep p >= min_p * max(p) (max(p) = 1 / total: the top element's exp is 1), renormalise
  const bool use_min_p = a.min_p > 0.f && a.min_p < 1.f;
  const float thr = use_min_p ? fmul(a.min_p, fdiv(1.f, total)) : 0.f;
  float total2 = 1.f;
  if (use_min_p) {
    float s2 = 0.f;
    for (int i = threadIdx.x; i < V; i += kSampleThreads) {
      const float q = fdiv(p[i], total);
      s2 = fadd(s2, q >= thr ? q : 0.f);
    }
    total2 = block_total(s2, sh);
  }
  for (int i = threadIdx.x; i < V; i += kSampleThreads) {
    float q = fdiv(p[i], total);
    if (use_min_p) q = q >= thr ? fdiv(q, total2) : 0.f;
    p[i] = q;
  }
  __syncthreads();

  int out;
  if (a.top_p < 1.f) {
    // nucleus: the descending prefix with cumulative mass <= floor(top_p * 2^52)
    const unsigned long long budget = __double2ull_rz(static_cast<double>(a.top_p) * kMassScale);
    const Crossing c1 = find_crossing(p, V, budget, sh, hmass, hcnt);
    unsigned long long n_mass;
    unsigned long long n_keep;
    if (c1.all_fit) {
      unsigned long long tot = 0;
      unsigned long long m = 0;
      for (int i = threadIdx.x; i < V; i += kSampleThreads) m += mass_of(p[i]);
      block_excl_scan(m, &tot, sh);
      n_mass = tot;
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
      for (int i = threadIdx.x; i < V; i += kSampleThreads) pm = fmaxf(pm, p[i]);
      pm = block_max(pm, sh);
      out = jth_with_key(p, V, __float_as_uint(pm), 0, sh);
    } else {
      unsigned long long target = __double2ull_rz(u * static_cast<double>(n_mass));
      if (target >= n_mass) target = n_mass - 1;
      const Crossing c2 = find_crossing(p, V, target, sh, hmass, hcnt);
      const unsigned long long mk = mass_of(__uint_as_float(c2.key));
      out = jth_with_key(p, V, c2.key, (target - c2.above) / mk, sh);
    }
  } else {
    unsigned long long tot = 0;
    unsigned long long m = 0;
    for (int i = threadIdx.x; i < V; i += kSampleThreads) m += mass_of(p[i]);
    block_excl_scan(m, &tot, sh);
    unsigned long long target = __double2ull_rz(u * static_cast<double>(tot));
    if (target >= tot) target = tot - 1;
    out = first_cum_above(p, V, target, sh);
  }
  if (threadIdx.x == 0) a.out[row] = out;
  grid_dep_launch();
}

}  // namespace

size_t sample_smem_bytes() {
  return static_cast<size_t>(kSampleWarps) * kBuckets * (sizeof(unsigned long long) + sizeof(unsigned));
}

cudaError_t sample_init_attrs() {
  return cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(sample_smem_bytes()));
}

cudaError_t launch_sample(const SampleArgs& a, int rows, bool pdl, cudaStream_t st) {
  if (rows < 1 || a.vocab < 1) return cudaErrorInvalidValue;
  cudaLaunchConfig_t c = {};
  c.gridDim = dim3(rows);
  c.blockDim = dim3(kSampleThreads);
  c.dynamicSmemBytes = sample_smem_bytes();
  c.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  c.attrs = attr;
  c.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&c, sample_kernel, a);
}

}  // namespace alm
