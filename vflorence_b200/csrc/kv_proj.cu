// Encoder K/V projection fused with the paged write (sm_100a tensor cores).
//
//   kv = hidden . w_kv^T (+ bias), hidden [T, K], w_kv [2*H*D, K] (the k rows, then the v rows),
//   then token t's k / v head h goes to cache[slot // bs, h, slot % bs, :] for slot =
//   slot_mapping[t] - the encoder half of ModelRunner._encode (vflorence/engine/model_runner.py:
//   248-259), which runs a GEMM per layer and then reshape_and_cache.
//
// One CTA (4 warps) computes one 128 x 128 tile of kv:
//   * warp 0, one thread: TMA loads of 128 x 64 tiles of hidden and w_kv (128-byte swizzle) into a
//     3-stage shared-memory ring paced by full / empty mbarriers;
//   * warp 1, one thread: per stage four tcgen05.mma (M 128, N 128, K 16, bf16 in, fp32 out)
//     into a 128-column TMEM accumulator, then tcgen05.commit to the stage's empty barrier, and
//     after the last stage to the accumulator barrier;
//   * all 4 warps: the epilogue - warp w reads TMEM lanes 32w..32w+31 (its tile rows) with
//     tcgen05.ld, adds the bias, rounds to bf16 and writes each token's 32-dim head slices
//     straight into its page (64 contiguous bytes per store group).
// Every wait is bounded (VFL_DEVERR_TIMEOUT); a CTA that gave up waits (bounded) for its copies
// and its MMAs, frees its TMEM and returns. Bad slots set VFL_DEVERR_SLOT and are skipped.
#include "common.cuh"

namespace vfl {
namespace {

constexpr int kBM = 128, kBN = 128, kBK = 64, kStages = 3;
constexpr int kTileBytes = kBM * kBK * 2;  // 16 KiB (A and B tiles alike)
constexpr int kTmemCols = 128;
constexpr int kSmemBytes = 1024 /* alignment slack */ + kStages * 2 * kTileBytes + 256 /* barriers */;

// tcgen05 instruction descriptor, kind::f16: f32 accumulator, bf16 A and B, both K-major,
// N = 128 (bits 17-22: N >> 3), M = 128 (bits 24-28: M >> 4)
constexpr uint32_t kInstrDesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                                ((uint32_t)(kBM >> 4) << 24);

// Shared-memory matrix descriptor of a K-major tile with the 128-byte swizzle: rows of 128 bytes,
// 8-row atoms 1024 bytes apart (SBO), leading offset field 1, descriptor version 1, layout 2.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

__device__ __forceinline__ void tma_load_tile(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(kInstrDesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct KvProjParams {
  const __nv_bfloat16* bias;  // [2 * H * D] or null
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  const int64_t* slots;
  int64_t num_tokens;
  int64_t num_blocks;
  int32_t k_dim;      // reduction length (hidden size), a multiple of 64
  int32_t heads;
  int32_t head_dim;   // a multiple of 32
  int32_t block_size;
  unsigned int* err;
};

__global__ void __launch_bounds__(128, 1) kv_proj_paged_kernel(const __grid_constant__ CUtensorMap amap,
                                                               const __grid_constant__ CUtensorMap bmap,
                                                               const KvProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t a_base = smem_u32(smem);
  const uint32_t b_base = a_base + kStages * kTileBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kStages * kTileBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* issued_slot = abort_flag + 1;
  int* consumed_slot = issued_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBN;
  const int64_t m0 = (int64_t)blockIdx.y * kBM;
  const int num_kb = p.k_dim / kBK;

  if (warp == 0) {  // TMEM: one warp allocates for the CTA
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    *issued_slot = 0;
    *consumed_slot = 0;
    fence_barrier_init();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- producer: TMA tiles of hidden (rows m0..) and w_kv (rows n0..), K step 64
    for (int kb = 0; kb < num_kb; ++kb) {
      const int s = kb % kStages;
      if (kb >= kStages && !mbar_wait_bounded(&empty[s], ((kb / kStages) - 1) & 1)) {
        report(p.err, VFL_DEVERR_TIMEOUT);
        *reinterpret_cast<volatile int*>(abort_flag) = 1;
        break;
      }
      if (*reinterpret_cast<volatile int*>(abort_flag)) break;
      mbar_arrive_expect_tx(&full[s], 2u * kTileBytes);
      tma_load_tile(a_base + s * kTileBytes, &amap, kb * kBK, (int)m0, &full[s]);
      tma_load_tile(b_base + s * kTileBytes, &bmap, kb * kBK, n0, &full[s]);
      *reinterpret_cast<volatile int*>(issued_slot) = kb + 1;
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer: four K-16 steps per stage (the descriptor start moves 32 bytes a step)
    for (int kb = 0; kb < num_kb; ++kb) {
      const int s = kb % kStages;
      if (!mbar_wait_bounded(&full[s], (kb / kStages) & 1)) {
        report(p.err, VFL_DEVERR_TIMEOUT);
        *reinterpret_cast<volatile int*>(abort_flag) = 1;
        break;
      }
      *reinterpret_cast<volatile int*>(consumed_slot) = kb + 1;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a = a_base + s * kTileBytes, b = b_base + s * kTileBytes;
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k)
        umma_bf16(tmem, smem_desc(a + k * 32), smem_desc(b + k * 32), (kb | k) != 0 ? 1u : 0u);
      umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
    }
    umma_commit(acc_full);  // arrives when every MMA issued above has completed
  }
  __syncwarp();

  // ---- epilogue: TMEM -> registers -> bias, bf16 -> pages
  const bool acc_ok = mbar_wait_bounded(acc_full, 0);
  if (!acc_ok) report(p.err, VFL_DEVERR_TIMEOUT);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const bool aborted = *reinterpret_cast<volatile int*>(abort_flag) != 0;
  const int row = warp * 32 + lane;
  const int64_t t = m0 + row;
  int64_t slot = -1;
  if (t < p.num_tokens) {
    slot = __ldg(p.slots + t);
    if (slot >= p.num_blocks * p.block_size) {
      report(p.err, VFL_DEVERR_SLOT);
      slot = -1;
    }
  }
  const int hd = p.heads * p.head_dim;
  if (acc_ok && !aborted) {
#pragma unroll 1
    for (int c0 = 0; c0 < kBN; c0 += 32) {
      uint32_t r[32];
      tmem_ld_32cols(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);  // every lane takes part
      const int f = n0 + c0;  // first feature of the chunk; a chunk lies in one head of k or v
      if (slot < 0 || f >= 2 * hd) continue;
      const bool is_v = f >= hd;
      const int within = is_v ? f - hd : f;
      const int h = within / p.head_dim, d0 = within - h * p.head_dim;
      const int64_t blk = slot / p.block_size, off = slot - blk * p.block_size;
      __nv_bfloat16* dst = (is_v ? p.v_cache : p.k_cache) +
                           (((blk * p.heads + h) * p.block_size + off) * p.head_dim + d0);
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float lo = __uint_as_float(r[2 * j]), hi = __uint_as_float(r[2 * j + 1]);
        if (p.bias != nullptr) {
          lo += __bfloat162float(p.bias[f + 2 * j]);
          hi += __bfloat162float(p.bias[f + 2 * j + 1]);
        }
        packed[j] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
                    ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
      }
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        d4[q] = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
    }
  }
  if (threadIdx.x == 0 && (aborted || !acc_ok)) {
    // copies issued but never consumed may still land in this CTA's shared memory: wait for
    // them (bounded) before the CTA exits
    const int issued = *reinterpret_cast<volatile int*>(issued_slot);
    for (int kb = *reinterpret_cast<volatile int*>(consumed_slot); kb < issued; ++kb)
      mbar_wait_bounded(&full[kb % kStages], (kb / kStages) & 1);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

int g_smem_done[kMaxDevices];

}  // namespace
}  // namespace vfl

using namespace vfl;

extern "C" int vfl_kv_proj_paged(const void* hidden, int64_t hidden_stride, const void* w_kv, const void* bias,
                                 void* k_cache, void* v_cache, const int64_t* slot_mapping, int64_t num_tokens,
                                 int32_t hidden_dim, int32_t num_heads, int32_t head_dim, int32_t block_size,
                                 int64_t num_blocks, void* stream) {
  if (num_tokens < 0 || num_tokens > (int64_t)65535 * kBM || hidden_dim <= 0 || hidden_dim % kBK != 0 ||
      hidden_dim > (1 << 20) || num_heads <= 0 || head_dim <= 0 || head_dim % 32 != 0 || block_size <= 0 ||
      num_blocks <= 0)
    return fail(VFL_ERR_INVALID_ARGUMENT,
                "kv_proj_paged: tokens %lld, hidden_dim %d (a multiple of 64), heads %d, head_dim %d (a multiple "
                "of 32), block_size %d, blocks %lld",
                (long long)num_tokens, hidden_dim, num_heads, head_dim, block_size, (long long)num_blocks);
  const int64_t n = 2LL * num_heads * head_dim;
  if (n % kBN != 0 || n > (1 << 20))
    return fail(VFL_ERR_UNSUPPORTED, "kv_proj_paged: 2 * heads * head_dim = %lld is not a multiple of %d",
                (long long)n, kBN);
  if (num_tokens == 0) return VFL_OK;
  if (!hidden || !w_kv || !k_cache || !v_cache || !slot_mapping)
    return fail(VFL_ERR_INVALID_ARGUMENT, "kv_proj_paged: NULL pointer");
  if (!aligned16(hidden) || !aligned16(w_kv) || !aligned16(k_cache) || !aligned16(v_cache) ||
      (hidden_stride * 2) % 16 != 0 || hidden_stride < hidden_dim)
    return fail(VFL_ERR_INVALID_ARGUMENT, "kv_proj_paged: pointers and the hidden row stride must be 16-byte aligned");
  CUtensorMap amap, bmap;
  int st = make_tensor_map_2d_bf16(hidden, (uint64_t)hidden_dim, (uint64_t)num_tokens, (uint64_t)hidden_stride * 2,
                                   kBK, kBM, &amap);
  if (st) return st;
  st = make_tensor_map_2d_bf16(w_kv, (uint64_t)hidden_dim, (uint64_t)n, (uint64_t)hidden_dim * 2, kBK, kBN, &bmap);
  if (st) return st;
  st = ensure_smem_attribute(reinterpret_cast<const void*>(&kv_proj_paged_kernel), kSmemBytes, g_smem_done);
  if (st) return st;
  KvProjParams p{};
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  p.slots = slot_mapping;
  p.num_tokens = num_tokens;
  p.num_blocks = num_blocks;
  p.k_dim = hidden_dim;
  p.heads = num_heads;
  p.head_dim = head_dim;
  p.block_size = block_size;
  st = device_error_word(&p.err);
  if (st) return st;
  dim3 grid((unsigned)(n / kBN), (unsigned)((num_tokens + kBM - 1) / kBM));
  kv_proj_paged_kernel<<<grid, 128, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(amap, bmap, p);
  return cuda_status(cudaGetLastError(), "kv_proj_paged launch");
}
