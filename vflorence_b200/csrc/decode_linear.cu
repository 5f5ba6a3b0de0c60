// Skinny linear layer of a decode step: y[m, n] = act(x[m, :] . w[n, :] + b[n]) for a few rows
// (m < rows <= 16) - the decoder's projections, feed-forward layers and vocabulary projection
// when a step feeds only a handful of sequences (vflorence/models/bart.py:106-146, :311-316,
// fp32 greedy decoding of BASELINE config 1). With so few rows the layer is a weight stream:
// every weight is used by `rows` multiply-adds, so the bound is HBM (4 bytes per fp32 weight).
//
// Work split: a CTA of 8 warps owns 32 output columns (4 per warp) of one K slice. It stages
// its rows' x[:, slice] in shared memory; each warp streams its 4 weight rows over the slice with
// 16-byte loads (lane l reads elements 4l..4l+3 of every 128-element chunk, so a warp's load of a
// row is one 512-byte segment), 2-4 chunks in flight per lane, multiply-adds into 4 x MR
// accumulators, then reduces them across lanes with a transposing butterfly (31 shuffles for 32
// values; lane j ends with the total of value j). When the columns alone give too few CTAs,
// K is split over a cluster of S <= 8 CTAs; the partial sums meet in distributed shared memory
// and each CTA of the cluster finishes an equal share of the tile, adding the S partials in a
// fixed order (results do not depend on timing). Bias and the exact GELU run in that epilogue.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace vfl {
namespace {

constexpr int kWarps = 8;
constexpr int kColsPerWarp = 4;
constexpr int kColsPerCta = kWarps * kColsPerWarp;  // 32
constexpr int kChunk = 128;                         // K elements per warp-wide load step
constexpr int kMaxRows = 16;
constexpr int kMaxSplits = 8;
constexpr int kMaxSmem = 64 * 1024;

struct DecodeLinearParams {
  const float* x;
  int64_t x_stride;
  const float* w;
  const float* bias;
  float* y;
  int64_t y_stride;
  int rows, n, k, kslice, act;
};

__device__ __forceinline__ float4 ldg_nc_f4(const float* p) {
  const uint4 v = ldg_nc_v4(p);
  return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
}

__device__ __forceinline__ float activate(float v, int act) {
  return act == VFL_ACT_GELU ? 0.5f * v * (1.f + erff(v * 0.70710678118654752f)) : v;
}

// Transposing reduction of NV (a power of two <= 32) values across the warp: on return v[0] holds,
// on lane l, the warp-wide total of value (l % NV).
template <int NV>
__device__ __forceinline__ void transpose_reduce(float* v, int lane) {
#pragma unroll
  for (int o = 16; o >= NV; o >>= 1)
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
#pragma unroll
  for (int o = NV / 2; o >= 1; o >>= 1) {
    const bool upper = lane & o;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float keep = upper ? v[i + o] : v[i];
      const float send = upper ? v[i] : v[i + o];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
}

template <int MR>
__global__ void __launch_bounds__(kWarps * 32) decode_linear_f32_kernel(DecodeLinearParams p) {
  constexpr int NV = kColsPerWarp * MR;      // accumulators per lane: value c * MR + m
  constexpr int U = MR >= 16 ? 2 : 4;        // chunks in flight per lane
  extern __shared__ float4 xs4[];            // [MR][kslice / 4]
  __shared__ float partial[kWarps * NV];     // this CTA's sums, read by the cluster (S > 1)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = gridDim.y;
  const int kslice = p.kslice, kq = kslice / 4;
  const int k0 = blockIdx.y * kslice;
  const int n0 = blockIdx.x * kColsPerCta + warp * kColsPerWarp;
  const float* wl = p.w + (size_t)n0 * p.k + k0 + lane * 4;
  const int iters = kslice / kChunk;
  // the first weight chunks go out before the rows are staged: their DRAM latency overlaps
  // the staging (the weights do not depend on it)
  float4 wv[U][kColsPerWarp];
#pragma unroll
  for (int u = 0; u < U; ++u)
#pragma unroll
    for (int c = 0; c < kColsPerWarp; ++c)
      wv[u][c] = u < iters ? ldg_nc_f4(wl + (size_t)c * p.k + u * kChunk) : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = threadIdx.x; i < MR * kq; i += kWarps * 32) {
    const int m = i / kq, c = i - m * kq;
    xs4[i] = m < p.rows ? *reinterpret_cast<const float4*>(p.x + m * p.x_stride + k0 + 4 * c)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();

  float acc[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) acc[i] = 0.f;
#pragma unroll 1
  for (int it0 = 0; it0 < iters; it0 += U) {
    if (it0 > 0) {
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int c = 0; c < kColsPerWarp; ++c)
          wv[u][c] = it0 + u < iters ? ldg_nc_f4(wl + (size_t)c * p.k + (it0 + u) * kChunk)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (it0 + u >= iters) break;
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        const float4 xv = xs4[m * kq + (it0 + u) * (kChunk / 4) + lane];
#pragma unroll
        for (int c = 0; c < kColsPerWarp; ++c) {
          float& a = acc[c * MR + m];
          a = fmaf(wv[u][c].x, xv.x, a);
          a = fmaf(wv[u][c].y, xv.y, a);
          a = fmaf(wv[u][c].z, xv.z, a);
          a = fmaf(wv[u][c].w, xv.w, a);
        }
      }
    }
  }

  // lane l: total of value l % 32 of each group of 32 values
  constexpr int G = NV > 32 ? NV / 32 : 1;
  constexpr int NG = NV > 32 ? 32 : NV;
#pragma unroll
  for (int g = 0; g < G; ++g) transpose_reduce<NG>(acc + g * NG, lane);

  if (S == 1) {  // the tile is complete: epilogue straight from the lanes
    if (lane < NG) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int v = g * NG + lane, c = v / MR, m = v - c * MR;
        if (m < p.rows) {
          const int n = n0 + c;
          const float b = p.bias != nullptr ? __ldg(p.bias + n) : 0.f;
          p.y[m * p.y_stride + n] = activate(acc[g * NG] + b, p.act);
        }
      }
    }
    return;
  }

  if (lane < NG) {
#pragma unroll
    for (int g = 0; g < G; ++g) partial[warp * NV + g * NG + lane] = acc[g * NG];
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();  // every CTA's partials are in its shared memory
  const int rank = static_cast<int>(cluster.block_rank());
  constexpr int E = kWarps * NV;
  const int per = E / S;
  for (int e = rank * per + threadIdx.x; e < (rank + 1) * per; e += kWarps * 32) {
    float t = 0.f;
    for (int s = 0; s < S; ++s) t += cluster.map_shared_rank(partial, s)[e];  // fixed order
    const int w = e / NV, v = e - w * NV, c = v / MR, m = v - c * MR;
    if (m < p.rows) {
      const int n = blockIdx.x * kColsPerCta + w * kColsPerWarp + c;
      const float b = p.bias != nullptr ? __ldg(p.bias + n) : 0.f;
      p.y[m * p.y_stride + n] = activate(t + b, p.act);
    }
  }
  cluster.sync();  // no CTA leaves while another still reads its partials
}

// K splits for a layer: the fewest that give every SM a CTA (where K allows), so the grid stays
// within one wave of two CTAs per SM and each CTA streams several chunks per warp, with the
// staged rows within the shared-memory budget. 0 when no split fits.
int choose_splits(int mr, int n, int k) {
  const int tiles = n / kColsPerCta;
  int s = 1;
  auto fits = [&](int sp) { return k % (sp * kChunk) == 0 && (size_t)mr * (k / sp) * 4 <= (size_t)kMaxSmem; };
  while (s < kMaxSplits && (tiles * s < kNumSMs || !fits(s)) && k % (2 * s * kChunk) == 0) s *= 2;
  return fits(s) ? s : 0;
}

template <int MR>
int launch(const DecodeLinearParams& p, int splits, cudaStream_t stream) {
  static int smem_done[kMaxDevices] = {};
  const int smem = MR * p.kslice * 4;
  auto kern = decode_linear_f32_kernel<MR>;
  int st = ensure_smem_attribute(reinterpret_cast<const void*>(kern), smem, smem_done);
  if (st) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n / kColsPerCta, splits, 1);
  cfg.blockDim = dim3(kWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, p), "decode_linear launch");
}

}  // namespace
}  // namespace vfl

using namespace vfl;

extern "C" int vfl_decode_linear_supported(int dtype, int rows, int n, int k) {
  if (dtype != VFL_DTYPE_F32 || rows < 1 || rows > kMaxRows || n <= 0 || k <= 0) return 0;
  if (n % kColsPerCta != 0 || k % kChunk != 0) return 0;
  return choose_splits(next_pow2(rows), n, k) > 0 ? 1 : 0;
}

extern "C" int vfl_decode_linear(const void* x, int64_t x_stride, const void* weight, const void* bias, void* y,
                                 int64_t y_stride, int32_t rows, int32_t n, int32_t k, int32_t dtype,
                                 int32_t activation, void* stream) {
  if (dtype != VFL_DTYPE_F32) return fail(VFL_ERR_UNSUPPORTED, "decode_linear: dtype %d (float32 only)", dtype);
  if (activation != VFL_ACT_NONE && activation != VFL_ACT_GELU)
    return fail(VFL_ERR_INVALID_ARGUMENT, "decode_linear: activation %d", activation);
  if (rows < 0 || n <= 0 || k <= 0) return fail(VFL_ERR_INVALID_ARGUMENT, "decode_linear: rows %d, n %d, k %d", rows, n, k);
  if (rows == 0) return VFL_OK;
  if (!vfl_decode_linear_supported(dtype, rows, n, k))
    return fail(VFL_ERR_UNSUPPORTED,
                "decode_linear: rows %d (1..16), n %d (a multiple of 32), k %d (a multiple of 128 whose "
                "slices fit shared memory)", rows, n, k);
  if (!x || !weight || !y) return fail(VFL_ERR_INVALID_ARGUMENT, "decode_linear: NULL pointer");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(y) || (bias && (reinterpret_cast<uintptr_t>(bias) & 3u)) ||
      x_stride % 4 || x_stride < k || y_stride < n)
    return fail(VFL_ERR_INVALID_ARGUMENT,
                "decode_linear: x, weight and y must be 16-byte aligned, x_stride a multiple of 4 >= k, "
                "y_stride >= n");
  const int mr = next_pow2(rows);
  const int splits = choose_splits(mr, n, k);
  DecodeLinearParams p{static_cast<const float*>(x), x_stride, static_cast<const float*>(weight),
                       static_cast<const float*>(bias), static_cast<float*>(y), y_stride, rows, n, k, k / splits,
                       activation};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (mr) {
    case 1: return launch<1>(p, splits, s);
    case 2: return launch<2>(p, splits, s);
    case 4: return launch<4>(p, splits, s);
    case 8: return launch<8>(p, splits, s);
    default: return launch<16>(p, splits, s);
  }
}
