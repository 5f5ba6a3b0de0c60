// bf16 linear layer of a decode step on the 5th-generation tensor cores:
//   y[m, n] = act(x[m, :] . w[n, :] + b[n]) for m < rows <= 256 (bf16 in, fp32 accumulate, bf16 out)
// - the decoder's projections and feed-forward layers (vflorence/models/bart.py:106-146) at the
// batch sizes of a decode step (128-256 rows). There the layer is small
// (1-8 MB of weights, K = 768-4096) and a library GEMM that walks K serially in 64-wide steps
// spends its time in latency: 6.5 us per layer for well under 1 us of HBM or tensor time.
//
// Here a CTA owns a 64-column tile for all rows (two 128-row accumulators in TMEM when rows > 128)
// and one K slice of at most 4 steps of 64 (8 for K = 4096): K is split over a thread-block
// cluster of up to 8 CTAs.
//   * warp 4, one thread: TMA loads (128-byte swizzle, no multicast) of the slice's x rows and
//     w rows into a ring of up to 4 stages paced by full / empty mbarriers;
//   * warp 5: allocates 128 TMEM columns; one thread issues tcgen05.mma (M 128, N 64, K 16) per
//     row half and K step, commits each stage to its empty barrier and the whole slice to the
//     accumulator barrier;
//   * warps 0-3 read the accumulators (tcgen05.ld, TMEM lane = row). Without a split they add
//     the bias (staged in shared memory), apply the exact GELU and store bf16. With one, each
//     row's fp32 partial goes with remote stores into a receive buffer of the CTA of the cluster
//     that finishes that row (an equal share of the rows each); after one cluster barrier every
//     CTA adds its rows' partials in rank order (results do not depend on timing), then bias,
//     GELU and one rounding to bf16. (Pulling the partials with remote loads instead cost twice
//     the time: each load waited out the cluster round trip.)
// Every mbarrier wait is bounded (VFL_DEVERR_TIMEOUT): a CTA that gives up stops issuing, skips
// its partials, waits (bounded) for its copies and MMAs, and still takes its cluster barriers,
// so its cluster never waits on it; TMEM is freed before exit.
#include <cooperative_groups.h>

#include "common.cuh"
#include "tcgen05.cuh"

namespace cg = cooperative_groups;

namespace vfl {
namespace {

constexpr int kBN = 64, kBK = 64, kHalfRows = 128;
constexpr int kMaxRingStages = 4;
constexpr int kTileX = kHalfRows * kBK * 2;  // 16 KiB: 128 rows x 64 bf16
constexpr int kTileW = kBN * kBK * 2;        // 8 KiB
constexpr int kThreads = 192;                // epilogue warps 0-3, producer warp 4, MMA warp 5
constexpr int kProducerWarp = 4, kMmaWarp = 5;
constexpr int kTmemCols = 2 * kBN;           // one 64-column accumulator per row half
constexpr int kMaxSplitsG = 8;
constexpr int kMaxRowsG = 256;
// kind::f16 instruction descriptor: f32 accumulator, bf16 A and B, both K-major, N = 64, M = 128
constexpr uint32_t kInstrDesc =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kHalfRows >> 4) << 24);

struct DecodeGemmParams {
  const __nv_bfloat16* bias;
  __nv_bfloat16* y;
  int64_t y_stride;
  int rows, n, kslice, halves, stages, act;
  int per;         // rows each CTA of a split cluster finishes (ceil(rows / splits))
  int recv_bytes;  // its receive buffer: splits x per rows of 64 fp32
  unsigned int* err;
};

struct GemmSmem {
  uint64_t full[kMaxRingStages], empty[kMaxRingStages];
  uint64_t acc_full;
  uint32_t tmem;
  int abort;
  int issued, consumed;  // K steps loaded by the producer / consumed by the MMA thread
  float bias[kBN];
};

__device__ __forceinline__ bool gemm_aborted(const GemmSmem& sh) {
  return *reinterpret_cast<const volatile int*>(&sh.abort);
}

__device__ __forceinline__ void gemm_give_up(GemmSmem& sh, unsigned int* err) {
  report(err, VFL_DEVERR_TIMEOUT);
  *reinterpret_cast<volatile int*>(&sh.abort) = 1;
}

__device__ __forceinline__ float gemm_act(float v, int act) {
  return act == VFL_ACT_GELU ? 0.5f * v * (1.f + erff(v * 0.70710678118654752f)) : v;
}

// Receive buffer of a split cluster: [source rank][owned row][16 float4], chunk c of a row stored
// at c ^ (row & 7) so that the lanes of a store phase (consecutive rows) hit distinct bank groups.
__device__ __forceinline__ int recv_index(int slot, int row, int c) { return slot * (kBN / 4) + (c ^ (row & 7)); }

// Cluster barrier in two halves: every thread arrives, and later waits for the whole cluster.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Shared memory: the stage ring, the receive buffer (split clusters), the barriers and bias.
__host__ __device__ constexpr int ring_bytes(int halves, int stages) { return stages * (halves * kTileX + kTileW); }
__host__ __device__ constexpr int smem_bytes(int halves, int stages, int recv_bytes) {
  return 1024 /* alignment */ + ring_bytes(halves, stages) + recv_bytes + (int)sizeof(GemmSmem);
}

__global__ void __launch_bounds__(kThreads, 1) decode_gemm_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                  const __grid_constant__ CUtensorMap wmap,
                                                                  const DecodeGemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stage_bytes = p.halves * kTileX + kTileW;
  const uint32_t ring = smem_u32(smem);  // stage s: x half 0, [x half 1], w
  float4* recv = reinterpret_cast<float4*>(smem + ring_bytes(p.halves, p.stages));
  GemmSmem& sh = *reinterpret_cast<GemmSmem*>(smem + ring_bytes(p.halves, p.stages) + p.recv_bytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBN;
  const int k0 = blockIdx.y * p.kslice;
  const int num_kb = p.kslice / kBK;
  const int S = gridDim.y;

  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    mbar_init(&sh.acc_full, 1);
    sh.abort = 0;
    sh.issued = sh.consumed = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < kBN) sh.bias[threadIdx.x] = p.bias != nullptr ? __bfloat162float(p.bias[n0 + threadIdx.x]) : 0.f;
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sh.tmem;
  if (S > 1) cluster_arrive_relaxed();  // this CTA has started; waited for before the first remote store

  if (warp == kProducerWarp) {
    if (lane == 0) {
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % p.stages;
        if (kb >= p.stages && !mbar_wait_bounded(&sh.empty[s], ((kb / p.stages) - 1) & 1)) {
          gemm_give_up(sh, p.err);
          break;
        }
        if (gemm_aborted(sh)) break;
        mbar_arrive_expect_tx(&sh.full[s], (uint32_t)stage_bytes);
        const uint32_t a = ring + s * stage_bytes;
        const int x = k0 + kb * kBK;
        tma_load_tile(a, &xmap, x, 0, &sh.full[s]);
        if (p.halves == 2) tma_load_tile(a + kTileX, &xmap, x, kHalfRows, &sh.full[s]);
        tma_load_tile(a + p.halves * kTileX, &wmap, x, n0, &sh.full[s]);
        *reinterpret_cast<volatile int*>(&sh.issued) = kb + 1;
      }
    }
    __syncwarp();
    if (S > 1) cluster_wait();
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % p.stages;
        if (!mbar_wait_bounded(&sh.full[s], (kb / p.stages) & 1)) {
          gemm_give_up(sh, p.err);
          break;
        }
        *reinterpret_cast<volatile int*>(&sh.consumed) = kb + 1;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a = ring + s * stage_bytes, wt = a + p.halves * kTileX;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t dw = smem_desc(wt + k * 32);
          const uint32_t acc_flag = (kb | k) != 0 ? 1u : 0u;
          umma_bf16(tmem, smem_desc(a + k * 32), dw, kInstrDesc, acc_flag);
          if (p.halves == 2) umma_bf16(tmem + (uint32_t)kBN, smem_desc(a + kTileX + k * 32), dw, kInstrDesc, acc_flag);
        }
        umma_commit(&sh.empty[s]);  // the stage is free once these MMAs have read it
      }
      umma_commit(&sh.acc_full);  // arrives once every MMA issued above has completed
    }
    __syncwarp();
    if (S > 1) cluster_wait();
  } else {
    // ---- warps 0-3: TMEM lanes 32w..32w+31 hold rows 32w..32w+31 of each row half
    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&sh.acc_full, 0));
    if (!ok && lane == 0) gemm_give_up(sh, p.err);
    const bool work = ok && !__any_sync(0xffffffffu, gemm_aborted(sh));
    if (S > 1) cluster_wait();  // every CTA of the cluster has started: its receive buffer exists
    if (work) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      cg::cluster_group cluster = cg::this_cluster();
      const int rank = static_cast<int>(blockIdx.y);
      for (int h = 0; h < p.halves; ++h) {
        const int r = h * kHalfRows + warp * 32 + lane;
        const uint32_t acc = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(h * kBN);
        uint32_t v[2][32];
        tmem_ld_32cols_issue(acc, v[0]);
        tmem_ld_32cols_issue(acc + 32u, v[1]);
        tmem_wait_ld();
        if (r >= p.rows) continue;
        if (S == 1) {  // the tile is complete: bias, activation, bf16, this lane's row
          uint4* dst = reinterpret_cast<uint4*>(p.y + (int64_t)r * p.y_stride + n0);
#pragma unroll
          for (int q = 0; q < kBN / 8; ++q) {
            uint32_t packed[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int c = q * 8 + 2 * j;
              const float lo = __uint_as_float(v[c >> 5][c & 31]) + sh.bias[c];
              const float hi = __uint_as_float(v[(c + 1) >> 5][(c + 1) & 31]) + sh.bias[c + 1];
              packed[j] = pack_bf16x2(gemm_act(lo, p.act), gemm_act(hi, p.act));
            }
            dst[q] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          }
        } else {  // the row's partial to the CTA that finishes it: slot [this rank][owned row]
          const int owner = r / p.per, local = r - owner * p.per;
          float4* dst = cluster.map_shared_rank(recv, owner);
          const int slot = rank * p.per + local;
#pragma unroll
          for (int c = 0; c < kBN / 4; ++c)
            dst[recv_index(slot, local, c)] =
                make_float4(__uint_as_float(v[c >> 3][(4 * c) & 31]), __uint_as_float(v[c >> 3][(4 * c + 1) & 31]),
                            __uint_as_float(v[c >> 3][(4 * c + 2) & 31]), __uint_as_float(v[c >> 3][(4 * c + 3) & 31]));
        }
      }
    }
  }
  __syncwarp();                          // converged warps for the .aligned cluster barrier
  if (S > 1) cluster_arrive_release();  // this CTA's partials are in their owners' buffers

  // ---- every MMA and copy of this CTA done (bounded), then the accumulators may be freed
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0 && gemm_aborted(sh)) {
    const int issued = *reinterpret_cast<volatile int*>(&sh.issued);
    for (int q = *reinterpret_cast<volatile int*>(&sh.consumed); q < issued; ++q)
      mbar_wait_bounded(&sh.full[q % p.stages], (q / p.stages) & 1);
    mbar_wait_bounded(&sh.acc_full, 0);
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
  if (S == 1) return;

  // ---- split K: this CTA's rows, the partials of ranks 0..S-1 added in that order
  cluster_wait();  // every CTA's stores into this buffer have landed
  const int rank = static_cast<int>(blockIdx.y);
  const int r_begin = rank * p.per, owned = min(p.rows, r_begin + p.per) - r_begin;
  for (int i = threadIdx.x; i < owned * (kBN / 4); i += kThreads) {
    const int local = i / (kBN / 4), c = i % (kBN / 4);
    float4 t = recv[recv_index(local, local, c)];
    for (int s = 1; s < S; ++s) {
      const float4 u = recv[recv_index(s * p.per + local, local, c)];
      t.x += u.x, t.y += u.y, t.z += u.z, t.w += u.w;
    }
    t.x += sh.bias[4 * c], t.y += sh.bias[4 * c + 1], t.z += sh.bias[4 * c + 2], t.w += sh.bias[4 * c + 3];
    *reinterpret_cast<uint2*>(p.y + (int64_t)(r_begin + local) * p.y_stride + n0 + 4 * c) =
        make_uint2(pack_bf16x2(gemm_act(t.x, p.act), gemm_act(t.y, p.act)),
                   pack_bf16x2(gemm_act(t.z, p.act), gemm_act(t.w, p.act)));
  }
}

// K splits: slices of at most 4 steps of 64 (at most 8 splits), whole steps each.
int gemm_splits(int k) {
  int s = 1;
  while (s < kMaxSplitsG && k / s > 4 * kBK && (k / (2 * s)) % kBK == 0 && k % (2 * s) == 0) s *= 2;
  return s;
}

}  // namespace

bool decode_gemm_supported(int rows, int n, int k) {
  return rows >= 1 && rows <= kMaxRowsG && n > 0 && n % kBN == 0 && k > 0 && k % kBK == 0 && n <= (1 << 22) &&
         k <= (1 << 16);
}

int launch_decode_gemm(const void* x, int64_t x_stride, const void* w, const void* bias, void* y, int64_t y_stride,
                       int rows, int n, int k, int act, cudaStream_t stream) {
  static int smem_done[kMaxDevices];
  const int splits = gemm_splits(k);
  const int kslice = k / splits;
  const int halves = rows > kHalfRows ? 2 : 1;
  const int kb = kslice / kBK;
  const int max_stages = splits > 1 ? 3 : kMaxRingStages;  // room for the receive buffer
  const int stages = kb < max_stages ? kb : max_stages;
  const int per = (rows + splits - 1) / splits;
  const int recv_bytes = splits > 1 ? splits * per * kBN * 4 : 0;
  CUtensorMap xmap, wmap;
  // rows past `rows` (up to the row half) read as zeros: the tensor map's outer extent is `rows`
  int st = make_tensor_map_2d_bf16(x, (uint64_t)k, (uint64_t)rows, (uint64_t)x_stride * 2, kBK, kHalfRows, &xmap);
  if (st) return st;
  st = make_tensor_map_2d_bf16(w, (uint64_t)k, (uint64_t)n, (uint64_t)k * 2, kBK, kBN, &wmap);
  if (st) return st;
  // the largest layout: two row halves, 3 stages and a full receive buffer, or 4 stages alone
  constexpr int kSmemMax = smem_bytes(2, 3, kMaxSplitsG * ((kMaxRowsG + kMaxSplitsG - 1) / kMaxSplitsG) * kBN * 4) >
                                   smem_bytes(2, kMaxRingStages, 0)
                               ? smem_bytes(2, 3, kMaxSplitsG * ((kMaxRowsG + kMaxSplitsG - 1) / kMaxSplitsG) * kBN * 4)
                               : smem_bytes(2, kMaxRingStages, 0);
  static_assert(kSmemMax <= 227 * 1024, "decode_gemm shared memory");
  st = ensure_smem_attribute(reinterpret_cast<const void*>(&decode_gemm_kernel), kSmemMax, smem_done);
  if (st) return st;
  unsigned int* err = nullptr;
  st = device_error_word(&err);
  if (st) return st;
  DecodeGemmParams p{static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(y), y_stride, rows, n,
                     kslice, halves, stages, act, per, recv_bytes, err};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n / kBN, splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes(halves, stages, recv_bytes);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, decode_gemm_kernel, xmap, wmap, p), "decode_gemm launch");
}

}  // namespace vfl
