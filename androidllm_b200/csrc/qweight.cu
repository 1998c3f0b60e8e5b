// Device repack of androidllm block-quant weights into the qtile layout, and
// a dequantizer that decodes the qtile layout back to fp16 rows (bit-exact
// against androidllm/quant.py:58-65; used to check the layout).
#include "kernels.cuh"
#include "qtile.cuh"
#include "repack.cuh"

namespace alm {
namespace {

// One thread per (tile, kb, lane): assemble that lane's fragment data.
__global__ void repack_kernel(SrcSet s, const int* __restrict__ dst_src_row, int bits, int n_tiles,
                              int k_blocks, int k_pad, int rec_u4, uint4* __restrict__ out) {
  const long long gid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long total = static_cast<long long>(n_tiles) * k_blocks * kWarp;
  if (gid >= total) return;
  const int lane = static_cast<int>(gid % kWarp);
  const int kb = static_cast<int>((gid / kWarp) % k_blocks);
  const int tile = static_cast<int>(gid / (static_cast<long long>(kWarp) * k_blocks));
  const int g = lane >> 2, t = lane & 3;
  const int d0 = dst_src_row[tile * 16 + g];
  const int d1 = dst_src_row[tile * 16 + g + 8];
  uint32_t words[16];
#pragma unroll
  for (int st = 0; st < 4; ++st) {
    const int c = kb * 64 + 16 * st + 2 * t;
    const int cols[4] = {c, c + 1, c + 8, c + 9};
    int r0[4], r1[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      r0[j] = fetch_code(s, d0, cols[j], bits, k_pad);
      r1[j] = fetch_code(s, d1, cols[j], bits, k_pad);
    }
    if (bits == 4) {
      // nibbles n0..n7 = (g,c) (g+8,c) (g,c+8) (g+8,c+8) (g,c+1) (g+8,c+1) (g,c+9) (g+8,c+9)
      const int order[8] = {r0[0], r1[0], r0[2], r1[2], r0[1], r1[1], r0[3], r1[3]};
      uint32_t w = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) w |= static_cast<uint32_t>((order[j] + 8) & 0xf) << (4 * j);
      words[st] = w;
    } else if (bits == 8) {
      uint32_t wg = 0, wg8 = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        wg |= static_cast<uint32_t>((r0[j] + 128) & 0xff) << (8 * j);
        wg8 |= static_cast<uint32_t>((r1[j] + 128) & 0xff) << (8 * j);
      }
      words[2 * st] = wg;
      words[2 * st + 1] = wg8;
    } else {
      words[4 * st + 0] = static_cast<uint32_t>(r0[0]) | (static_cast<uint32_t>(r0[1]) << 16);
      words[4 * st + 1] = static_cast<uint32_t>(r1[0]) | (static_cast<uint32_t>(r1[1]) << 16);
      words[4 * st + 2] = static_cast<uint32_t>(r0[2]) | (static_cast<uint32_t>(r0[3]) << 16);
      words[4 * st + 3] = static_cast<uint32_t>(r1[2]) | (static_cast<uint32_t>(r1[3]) << 16);
    }
  }
  const int nvec = bits == 4 ? 1 : bits == 8 ? 2 : 4;
  for (int v = 0; v < nvec; ++v) {
    const size_t idx = (static_cast<size_t>(tile) * k_blocks + kb) * rec_u4 + v * kWarp + lane;
    out[idx] = make_uint4(words[4 * v], words[4 * v + 1], words[4 * v + 2], words[4 * v + 3]);
  }
}

// One thread per (tile, kb, scale set, g): half2 {scale(row g), scale(row g+8)}
// written after the codes of record (tile, kb).
__global__ void repack_scales_kernel(SrcSet s, const int* __restrict__ dst_src_row, int n_tiles, int k_blocks,
                                     int block, int sets, int src_nsb, int vec, int rec_u4, uint4* __restrict__ out) {
  const long long gid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (gid >= static_cast<long long>(n_tiles) * k_blocks * sets * 8) return;
  const int g = static_cast<int>(gid & 7);
  const int set = static_cast<int>((gid >> 3) % sets);
  const int kb = static_cast<int>((gid >> 3) / sets % k_blocks);
  const int tile = static_cast<int>((gid >> 3) / sets / k_blocks);
  const int sbk = block == 32 ? 2 * kb + set : (kb * 64) / block;   // source scale block
  half v[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int desc = dst_src_row[tile * 16 + g + 8 * h];
    if (desc < 0 || sbk >= src_nsb) {
      v[h] = __ushort_as_half(0);
    } else {
      v[h] = s.scale[desc >> 24][static_cast<size_t>(desc & 0xffffff) * src_nsb + sbk];
    }
  }
  half2* sc = reinterpret_cast<half2*>(out + (static_cast<size_t>(tile) * k_blocks + kb) * rec_u4 + vec * kWarp);
  sc[set * 8 + g] = __halves2half2(v[0], v[1]);
}

// Decode the qtile layout back to fp16 rows (out: n_rows x k_real).
template <int BITS>
__global__ void dequant_kernel(QTile w, half* __restrict__ out) {
  const long long gid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long total = static_cast<long long>(w.n_tiles) * w.k_blocks * kWarp;
  if (gid >= total) return;
  const int lane = static_cast<int>(gid % kWarp);
  const int kb = static_cast<int>((gid / kWarp) % w.k_blocks);
  const int tile = static_cast<int>(gid / (static_cast<long long>(kWarp) * w.k_blocks));
  const int g = lane >> 2, t = lane & 3;
  constexpr int V = QTileTraits<BITS>::kVec;
  const uint4* rec = qtile_record(w, tile, kb);
  uint4 wd[V];
#pragma unroll
  for (int v = 0; v < V; ++v) wd[v] = rec[v * kWarp + lane];
#pragma unroll
  for (int st = 0; st < 4; ++st) {
    half2 sg = __float2half2_rn(1.f), sg8 = sg;
    if (BITS != 16) {
      const int set = (w.sb == 2 && st >= 2) ? 1 : 0;
      const half2 sc = reinterpret_cast<const half2*>(rec + V * kWarp)[set * 8 + g];
      sg = __low2half2(sc);
      sg8 = __high2half2(sc);
    }
    uint32_t a0, a1, a2, a3;
    decode_step<BITS>(wd, st, sg, sg8, a0, a1, a2, a3);
    const int c = kb * 64 + 16 * st + 2 * t;
    const int r0 = tile * 16 + g, r1 = r0 + 8;
    const uint32_t regs[4] = {a0, a1, a2, a3};
    const int rows[4] = {r0, r1, r0, r1};
    const int cols[4] = {c, c, c + 8, c + 8};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const half2 hv = u2h(regs[j]);
      if (rows[j] < w.n_rows) {
        const size_t base = static_cast<size_t>(rows[j]) * w.k_real;
        if (cols[j] < w.k_real) out[base + cols[j]] = __low2half(hv);
        if (cols[j] + 1 < w.k_real) out[base + cols[j] + 1] = __high2half(hv);
      }
    }
  }
}

}  // namespace

cudaError_t launch_repack(const void* const* src, const half* const* src_scales, int n_src,
                          const int* dst_src_row, QTile& w, uint4* data, int k_pad, cudaStream_t st) {
  if (n_src < 1 || n_src > 3) return cudaErrorInvalidValue;
  SrcSet s{};
  for (int i = 0; i < n_src; ++i) {
    s.data[i] = static_cast<const uint8_t*>(src[i]);
    s.scale[i] = src_scales ? src_scales[i] : nullptr;
  }
  const long long total = static_cast<long long>(w.n_tiles) * w.k_blocks * kWarp;
  const int threads = 256;
  repack_kernel<<<static_cast<unsigned>((total + threads - 1) / threads), threads, 0, st>>>(
      s, dst_src_row, w.bits, w.n_tiles, w.k_blocks, k_pad, w.rec_u4, data);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || w.bits == 16) return e;
  const int vec = w.bits == 4 ? 1 : 2;
  const long long n = static_cast<long long>(w.n_tiles) * w.k_blocks * w.sb * 8;
  repack_scales_kernel<<<static_cast<unsigned>((n + threads - 1) / threads), threads, 0, st>>>(
      s, dst_src_row, w.n_tiles, w.k_blocks, w.block, w.sb, k_pad / w.block, vec, w.rec_u4, data);
  return cudaGetLastError();
}

cudaError_t launch_dequant(const QTile& w, half* out, cudaStream_t st) {
  const long long total = static_cast<long long>(w.n_tiles) * w.k_blocks * kWarp;
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((total + threads - 1) / threads);
  if (w.bits == 4) dequant_kernel<4><<<blocks, threads, 0, st>>>(w, out);
  else if (w.bits == 8) dequant_kernel<8><<<blocks, threads, 0, st>>>(w, out);
  else dequant_kernel<16><<<blocks, threads, 0, st>>>(w, out);
  return cudaGetLastError();
}

}  // namespace alm
