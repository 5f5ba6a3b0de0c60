// bf16 linear layer of a decode step on the 5th-generation tensor cores:
//   y[m, n] = act(x[m, :] . w[n, :] + b[n]) for m < rows <= 256 (bf16 in, fp32 accumulate, bf16 out)
// - the decoder's projections and feed-forward layers (vflorence/models/bart.py:106-146) at the
// batch sizes of a decode step (128-256 rows). There the layer is small
// (1-8 MB of weights, K = 768-4096) and a library GEMM that walks K serially in 64-wide steps
// spends its time in latency: 6.5 us per layer for well under 1 us of HBM or tensor time.
//
// Here a CTA owns a 64-column tile for all rows (two 128-row accumulators in TMEM when rows > 128)
// and one K slice; where the columns alone give fewer CTAs than SMs, K is split over a thread-
// block cluster of up to 8 CTAs, so each CTA has only 2-8 K steps of 64 to do:
//   * warp 4, one thread: TMA loads (128-byte swizzle, no multicast) of the slice's x rows and
//     w rows into a ring of up to 4 stages paced by full / empty mbarriers;
//   * warp 5: allocates 128 TMEM columns; one thread issues tcgen05.mma (M 128, N 64, K 16) per
//     row half and K step, commits each stage to its empty barrier and the whole slice to the
//     accumulator barrier;
//   * warps 0-3 read the accumulators (tcgen05.ld, TMEM lane = row) into the freed ring as fp32
//     partials; the cluster meets in distributed shared memory and each CTA finishes an equal
//     share of the tile's rows, adding the partials in a fixed order (results do not depend on
//     timing), then bias and the exact GELU, one rounding to bf16.
// Every mbarrier wait is bounded (VFL_DEVERR_TIMEOUT): a CTA that gives up stops issuing, skips
// its partials, waits (bounded) for its copies and MMAs, and still takes both cluster barriers,
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
  unsigned int* err;
};

struct GemmSmem {
  uint64_t full[kMaxRingStages], empty[kMaxRingStages];
  uint64_t acc_full;
  uint32_t tmem;
  int abort;
  int issued, consumed;  // K steps loaded by the producer / consumed by the MMA thread
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

// fp32 partials of the tile: row r's 16 float4 chunks, chunk c stored at c ^ (r & 7) so that the
// 8 lanes of a store phase (consecutive rows) hit distinct 16-byte bank groups
__device__ __forceinline__ int partial_index(int r, int c) { return r * (kBN / 4) + (c ^ (r & 7)); }

// Shared memory: the ring (reused for the fp32 partials once every MMA has read it), then the
// barriers. Host and device agree on the offsets.
__host__ __device__ constexpr int ring_bytes(int halves, int stages) { return stages * (halves * kTileX + kTileW); }
__host__ __device__ constexpr int partial_bytes(int halves) { return halves * kHalfRows * kBN * 4; }
__host__ __device__ constexpr int region_bytes(int halves, int stages) {
  return ring_bytes(halves, stages) > partial_bytes(halves) ? ring_bytes(halves, stages) : partial_bytes(halves);
}
__host__ __device__ constexpr int smem_bytes(int halves, int stages) {
  return 1024 /* alignment */ + region_bytes(halves, stages) + 256;
}

__global__ void __launch_bounds__(kThreads, 1) decode_gemm_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                  const __grid_constant__ CUtensorMap wmap,
                                                                  const DecodeGemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stage_bytes = p.halves * kTileX + kTileW;
  const uint32_t ring = smem_u32(smem);  // stage s: x half 0, [x half 1], w
  float4* partial = reinterpret_cast<float4*>(smem);  // the ring, once every MMA has completed
  GemmSmem& sh = *reinterpret_cast<GemmSmem*>(smem + region_bytes(p.halves, p.stages));
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
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sh.tmem;

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
  } else {
    // ---- warps 0-3: TMEM lanes 32w..32w+31 hold rows 32w..32w+31 of each row half
    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&sh.acc_full, 0));
    if (!ok && lane == 0) gemm_give_up(sh, p.err);
    if (ok && !__any_sync(0xffffffffu, gemm_aborted(sh))) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      for (int h = 0; h < p.halves; ++h) {
        const int r = h * kHalfRows + warp * 32 + lane;
        const uint32_t acc = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(h * kBN);
        uint32_t v[2][32];
        tmem_ld_32cols_issue(acc, v[0]);
        tmem_ld_32cols_issue(acc + 32u, v[1]);
        tmem_wait_ld();
        if (S == 1) {  // the tile is complete: bias, activation, bf16, this lane's row
          if (r < p.rows) {
            uint4* dst = reinterpret_cast<uint4*>(p.y + (int64_t)r * p.y_stride + n0);
#pragma unroll
            for (int q = 0; q < kBN / 8; ++q) {
              uint32_t packed[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int c = q * 8 + 2 * j;
                float lo = __uint_as_float(v[c >> 5][c & 31]), hi = __uint_as_float(v[(c + 1) >> 5][(c + 1) & 31]);
                if (p.bias != nullptr) {
                  lo += __bfloat162float(p.bias[n0 + c]);
                  hi += __bfloat162float(p.bias[n0 + c + 1]);
                }
                packed[j] = pack_bf16x2(gemm_act(lo, p.act), gemm_act(hi, p.act));
              }
              dst[q] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            }
          }
        } else {  // this CTA's partial sums for the cluster
#pragma unroll
          for (int c = 0; c < kBN / 4; ++c)
            partial[partial_index(r, c)] =
                make_float4(__uint_as_float(v[c >> 3][(4 * c) & 31]), __uint_as_float(v[c >> 3][(4 * c + 1) & 31]),
                            __uint_as_float(v[c >> 3][(4 * c + 2) & 31]), __uint_as_float(v[c >> 3][(4 * c + 3) & 31]));
        }
      }
    }
  }

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

  // ---- split K: each CTA of the cluster reduces an equal share of the rows, partials in rank order
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();  // every CTA's partials are in its shared memory (taken on every path)
  const int rank = static_cast<int>(cluster.block_rank());
  const int per = (p.rows + S - 1) / S;
  const int r_begin = rank * per, r_end = min(p.rows, r_begin + per);
  for (int i = threadIdx.x; i < (r_end - r_begin) * (kBN / 4); i += kThreads) {
    const int r = r_begin + i / (kBN / 4), c = i % (kBN / 4);
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < S; ++s) {
      const float4 v = cluster.map_shared_rank(partial, s)[partial_index(r, c)];
      t.x += v.x, t.y += v.y, t.z += v.z, t.w += v.w;
    }
    const int n = n0 + 4 * c;
    if (p.bias != nullptr) {
      t.x += __bfloat162float(p.bias[n]), t.y += __bfloat162float(p.bias[n + 1]);
      t.z += __bfloat162float(p.bias[n + 2]), t.w += __bfloat162float(p.bias[n + 3]);
    }
    *reinterpret_cast<uint2*>(p.y + (int64_t)r * p.y_stride + n) =
        make_uint2(pack_bf16x2(gemm_act(t.x, p.act), gemm_act(t.y, p.act)),
                   pack_bf16x2(gemm_act(t.z, p.act), gemm_act(t.w, p.act)));
  }
  cluster.sync();  // no CTA leaves while another still reads its partials
}

// K splits: the fewest that give every SM a CTA where K allows (slices of whole 64-wide steps).
int gemm_splits(int n, int k) {
  const int tiles = n / kBN;
  int s = 1;
  while (s < kMaxSplitsG && tiles * s < kNumSMs && (k / (2 * s)) % kBK == 0 && k % (2 * s) == 0) s *= 2;
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
  const int splits = gemm_splits(n, k);
  const int kslice = k / splits;
  const int halves = rows > kHalfRows ? 2 : 1;
  const int kb = kslice / kBK;
  const int stages = kb < kMaxRingStages ? kb : kMaxRingStages;
  CUtensorMap xmap, wmap;
  // rows past `rows` (up to the row half) read as zeros: the tensor map's outer extent is `rows`
  int st = make_tensor_map_2d_bf16(x, (uint64_t)k, (uint64_t)rows, (uint64_t)x_stride * 2, kBK, kHalfRows, &xmap);
  if (st) return st;
  st = make_tensor_map_2d_bf16(w, (uint64_t)k, (uint64_t)n, (uint64_t)k * 2, kBK, kBN, &wmap);
  if (st) return st;
  const int smem = smem_bytes(2, kMaxRingStages);
  st = ensure_smem_attribute(reinterpret_cast<const void*>(&decode_gemm_kernel), smem, smem_done);
  if (st) return st;
  unsigned int* err = nullptr;
  st = device_error_word(&err);
  if (st) return st;
  DecodeGemmParams p{static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(y), y_stride, rows, n,
                     kslice, halves, stages, act, err};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n / kBN, splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes(halves, stages);
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
