// Encoder K/V projection fused with the paged write (sm_100a tensor cores).
//
//   kv = hidden . w_kv^T (+ bias), hidden [T, K], w_kv [2*H*D, K] (the k rows, then the v rows),
//   then token t's k / v head h goes to cache[slot // bs, h, slot % bs, :] for slot =
//   slot_mapping[t] - the encoder half of ModelRunner._encode (vflorence/engine/model_runner.py:
//   248-259), which runs a GEMM per layer and then reshape_and_cache.
//
// Two persistent, warp-specialised kernels. From 6144 tokens (with a 256-multiple feature
// count) a 2-SM kernel (cta_group::2, further below) walks 256 x 256 tiles with a pair of CTAs;
// otherwise one CTA per SM walks 128 x BN output tiles (BN = 256 features where the feature
// count allows, else 128). Features run fastest, so consecutive tiles reuse the same hidden rows
// from L2. The one-CTA kernel:
//   * warp 4, one thread: TMA loads of 128 x 64 tiles of hidden and w_kv (128-byte swizzle) into
//     a 4-stage shared-memory ring paced by full / empty mbarriers, running ahead across tiles;
//   * warp 5: allocates 2 x BN TMEM columns (two fp32 accumulators); one thread issues, per
//     stage, four tcgen05.mma (M 128, N BN, K 16, bf16 in, fp32 out) and tcgen05.commit to
//     the stage's empty barrier, and after a tile's last stage to the accumulator's full barrier;
//   * warps 0-3: the epilogue of tile i (tcgen05.ld of TMEM lanes 32w..32w+31 = the tile's
//     rows, bias, bf16, each token's 32-dim head slices stored straight into its page) while the
//     tensor cores already accumulate tile i+1 into the other accumulator.
// Every wait is bounded (VFL_DEVERR_TIMEOUT): a CTA that gave up stops issuing, waits (bounded)
// for its copies and its MMAs, frees its TMEM and returns. Bad slots set VFL_DEVERR_SLOT.
#include "common.cuh"

namespace vfl {
namespace {

constexpr int kBM = 128, kBK = 64, kStages = 4;
constexpr int kTileA = kBM * kBK * 2;                  // 16 KiB
constexpr int kEpilogueWarps = 4;
constexpr int kThreads = (kEpilogueWarps + 2) * 32;   // + producer warp + MMA warp
constexpr int kProducerWarp = 4, kMmaWarp = 5;

// Tile width BN (output features): 256 where the feature count allows (a third less L2 traffic
// per flop than 128), else 128.
template <int BN>
struct KvTile {
  static constexpr int kTileB = BN * kBK * 2;
  static constexpr int kStageBytes = kTileA + kTileB;
  static constexpr int kAccCols = BN;          // one fp32 accumulator: BN TMEM columns
  static constexpr int kTmemCols = 2 * BN;     // double-buffered
  static constexpr int kSmemBytes = 1024 /* alignment slack */ + kStages * kStageBytes + 256 /* barriers */;
  // tcgen05 instruction descriptor, kind::f16: f32 accumulator, bf16 A and B, both K-major,
  // N = BN (bits 17-22: N >> 3), M = 128 (bits 24-28: M >> 4)
  static constexpr uint32_t kInstrDesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                         ((uint32_t)(kBM >> 4) << 24);
};

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

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Issues the load of 32 TMEM columns (32 lanes x 32 x 32 bits) into r; r is valid after
// tmem_wait_ld().
__device__ __forceinline__ void tmem_ld_32cols_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

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
  int32_t n_tiles;    // output feature tiles (2 * H * D / 128)
  int32_t tiles;      // n_tiles x token tiles
  unsigned int* err;
};

// One warp's share of a tile's epilogue: its 32 rows (TMEM lanes of `acc`, this lane's token at
// `slot`, -1 = skip) x BN features from n0: fp32 accumulators + bias -> bf16, each 32-feature
// chunk (one head slice of k or v) stored as 64 contiguous bytes in the token's page. The next
// chunk's TMEM load is in flight while a chunk is converted and stored; the chunk's 32 bias
// values come in with one load per lane and reach every lane by shuffles.
template <int BN>
__device__ __forceinline__ void store_rows(uint32_t acc, int n0, int64_t slot, const KvProjParams& p, int lane) {
  const int hd = p.heads * p.head_dim;
  const int64_t blk = slot / p.block_size, off = slot - blk * p.block_size;
  uint32_t r[2][32];
  tmem_ld_32cols_issue(acc, r[0]);  // every lane takes part in the TMEM loads and the shuffles
#pragma unroll
  for (int c = 0; c < BN / 32; ++c) {
    tmem_wait_ld();
    if (c + 1 < BN / 32) tmem_ld_32cols_issue(acc + (uint32_t)((c + 1) * 32), r[(c + 1) & 1]);
    const uint32_t(&v)[32] = r[c & 1];
    const int f = n0 + c * 32;  // first feature of the chunk; a chunk lies in one head of k or v
    const float bias_lane = p.bias != nullptr ? __bfloat162float(p.bias[f + lane]) : 0.f;
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float lo = __uint_as_float(v[2 * j]) + __shfl_sync(0xffffffffu, bias_lane, 2 * j);
      const float hi = __uint_as_float(v[2 * j + 1]) + __shfl_sync(0xffffffffu, bias_lane, 2 * j + 1);
      packed[j] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
                  ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
    }
    if (slot < 0) continue;
    const bool is_v = f >= hd;
    const int within = is_v ? f - hd : f;
    const int h = within / p.head_dim, d0 = within - h * p.head_dim;
    uint4* d4 = reinterpret_cast<uint4*>((is_v ? p.v_cache : p.k_cache) +
                                         (((blk * p.heads + h) * p.block_size + off) * p.head_dim + d0));
#pragma unroll
    for (int qq = 0; qq < 4; ++qq)
      d4[qq] = make_uint4(packed[4 * qq], packed[4 * qq + 1], packed[4 * qq + 2], packed[4 * qq + 3]);
  }
}

struct KvSmem {  // after the stage ring
  uint64_t full[kStages], empty[kStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem;
  int abort;
  int issued, consumed;  // k-block loads issued by the producer / consumed by the MMA thread
};

__device__ __forceinline__ bool aborted(const KvSmem& sh) { return *reinterpret_cast<const volatile int*>(&sh.abort); }

__device__ __forceinline__ void give_up(KvSmem& sh, unsigned int* err) {
  report(err, VFL_DEVERR_TIMEOUT);
  *reinterpret_cast<volatile int*>(&sh.abort) = 1;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) kv_proj_paged_kernel(const __grid_constant__ CUtensorMap amap,
                                                                   const __grid_constant__ CUtensorMap bmap,
                                                                   const KvProjParams p) {
  using Tile = KvTile<BN>;
  constexpr int kBN = BN, kStageBytes = Tile::kStageBytes, kAccCols = Tile::kAccCols, kTmemCols = Tile::kTmemCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t ring = smem_u32(smem);  // stage s: A tile at ring + s * kStageBytes, B tile after it
  KvSmem& sh = *reinterpret_cast<KvSmem*>(smem + kStages * kStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_kb = p.k_dim / kBK;

  if (warp == kMmaWarp) {  // TMEM: one warp allocates for the CTA
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.acc_full[b], 1);
      mbar_init(&sh.acc_empty[b], kEpilogueWarps);
    }
    mbar_init(&sh.mma_done, 1);
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
      int q = 0;  // k-block loads across this CTA's tiles
      for (int tile = blockIdx.x; tile < p.tiles && !aborted(sh); tile += gridDim.x) {
        const int n0 = (tile % p.n_tiles) * kBN;
        const int m0 = (tile / p.n_tiles) * kBM;
        for (int kb = 0; kb < num_kb; ++kb, ++q) {
          const int s = q % kStages;
          if (q >= kStages && !mbar_wait_bounded(&sh.empty[s], ((q / kStages) - 1) & 1)) {
            give_up(sh, p.err);
            break;
          }
          if (aborted(sh)) break;
          mbar_arrive_expect_tx(&sh.full[s], (uint32_t)kStageBytes);
          const uint32_t a = ring + s * kStageBytes;
          tma_load_tile(a, &amap, kb * kBK, m0, &sh.full[s]);
          tma_load_tile(a + kTileA, &bmap, kb * kBK, n0, &sh.full[s]);
          *reinterpret_cast<volatile int*>(&sh.issued) = q + 1;
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      int q = 0, i = 0;  // k-blocks consumed, tiles accumulated
      for (int tile = blockIdx.x; tile < p.tiles && !aborted(sh); tile += gridDim.x, ++i) {
        const int b = i & 1;
        // the epilogue must have emptied this accumulator (used two tiles ago)
        if (i >= 2 && !mbar_wait_bounded(&sh.acc_empty[b], ((i >> 1) - 1) & 1)) {
          give_up(sh, p.err);
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + (uint32_t)(b * kAccCols);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++q) {
          const int s = q % kStages;
          if (!mbar_wait_bounded(&sh.full[s], (q / kStages) & 1)) {
            give_up(sh, p.err);
            ok = false;
            break;
          }
          *reinterpret_cast<volatile int*>(&sh.consumed) = q + 1;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a = ring + s * kStageBytes, bt = a + kTileA;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16(acc, smem_desc(a + k * 32), smem_desc(bt + k * 32), Tile::kInstrDesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&sh.empty[s]);  // the stage is free once these MMAs have read it
        }
        if (!ok) break;
        umma_commit(&sh.acc_full[b]);  // the tile's accumulator is complete
      }
      umma_commit(&sh.mma_done);  // arrives once every MMA issued above has completed
    }
  } else {
    // ---- epilogue warps 0-3: TMEM lanes 32w..32w+31 are rows 32w..32w+31 of the tile
    int i = 0;
    for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, ++i) {
      const int b = i & 1;
      // warp-uniform: the tcgen05.ld below needs every lane
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&sh.acc_full[b], (i >> 1) & 1))) {
        give_up(sh, p.err);
        break;
      }
      if (__any_sync(0xffffffffu, aborted(sh))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int n0 = (tile % p.n_tiles) * kBN;
      const int64_t t = (int64_t)(tile / p.n_tiles) * kBM + warp * 32 + lane;
      int64_t slot = -1;
      if (t < p.num_tokens) {
        slot = __ldg(p.slots + t);
        if (slot >= p.num_blocks * p.block_size) {
          report(p.err, VFL_DEVERR_SLOT);
          slot = -1;
        }
      }
      const uint32_t acc = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * kAccCols);
      store_rows<kBN>(acc, n0, slot, p, lane);
      // this warp has its rows in registers: the accumulator may take the tile after next
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.acc_empty[b]);
    }
  }

  // ---- teardown: every issued MMA done, every issued copy landed, then TMEM freed
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!mbar_wait_bounded(&sh.mma_done, 0)) report(p.err, VFL_DEVERR_TIMEOUT);
    const int issued = *reinterpret_cast<volatile int*>(&sh.issued);
    for (int q = *reinterpret_cast<volatile int*>(&sh.consumed); q < issued; ++q)
      mbar_wait_bounded(&sh.full[q % kStages], (q / kStages) & 1);
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------------------------
// 2-SM variant: a cluster of two CTAs on two SMs computes 256 x 256 tiles with tcgen05.mma
// .cta_group::2 (M 256 = 128 rows per CTA, N 256 = 128 features' w_kv rows per CTA). Each SM
// stages 32 KiB per k-step instead of 48 KiB for the same tensor work (the L2 -> SM fill is what
// bounds the one-CTA kernel), so the ring is 6 stages deep.
//   * both CTAs, warp 4: TMA loads of its own hidden rows and w_kv rows; every copy completes on
//     the leader's (rank 0) full barrier, where the leader's producer alone arrives, expecting
//     both CTAs' bytes (a remote arrival with cluster-scope release would wait on the producer's
//     copies in flight, one round trip per stage);
//   * leader, warp 5, one thread: the MMAs, then tcgen05.commit to the stage's empty barrier of
//     each CTA (two plain commits), to each CTA's accumulator-full barrier after a tile, and to
//     each CTA's done barrier at the end;
//   * both CTAs, warps 0-3: the epilogue of the CTA's 128 rows x 256 features from its own TMEM,
//     then one arrival per warp on the leader's accumulator-empty barrier.
// Every wait is bounded; a CTA that gives up raises the abort flag of both CTAs.

constexpr int kPairStages = 6;
constexpr int kPairTileA = 128 * kBK * 2;                      // this CTA's 128 hidden rows
constexpr int kPairTileB = 128 * kBK * 2;                      // this CTA's 128 w_kv rows
constexpr int kPairStageBytes = kPairTileA + kPairTileB;       // 32 KiB
constexpr int kPairBM = 256, kPairBN = 256;                    // the pair's output tile
constexpr int kPairTmemCols = 512;                             // two 256-column fp32 accumulators
constexpr int kPairSmemBytes = 1024 + kPairStages * kPairStageBytes + 256;
// kind::f16, f32 accumulator, bf16 A and B, both K-major, N = 256, M = 256 (the pair)
constexpr uint32_t kPairInstrDesc =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kPairBN >> 3) << 17) | ((uint32_t)(kPairBM >> 4) << 24);
// the pair kernel pays from about 6K tokens (measured on B200 against the one-CTA kernel: slower
// at 2K, even at 4K, faster at 8K and at 50K); below it the one-CTA kernel's 128-row tiles keep
// more SMs busy
constexpr int64_t kPairMinTokens = 6144;

struct PairSmem {  // after the stage ring
  uint64_t full[kPairStages], empty[kPairStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem;
  int abort;
  int issued, consumed;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// This CTA's shared-memory address `addr` mapped to the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrival on a barrier of either CTA of the pair (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Counts `bytes` as landed on this CTA's barrier `bar` (for copies that were expected but never
// issued).
__device__ __forceinline__ void mbar_complete_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.complete_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// A TMA copy into this CTA's shared memory whose completion is counted on `bar`, a barrier of
// either CTA of the pair (shared::cluster address).
__device__ __forceinline__ void tma_load_tile_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` (a barrier of either CTA) once every MMA this thread issued has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void give_up_pair(PairSmem& sh, uint32_t peer_abort, unsigned int* err) {
  report(err, VFL_DEVERR_TIMEOUT);
  *reinterpret_cast<volatile int*>(&sh.abort) = 1;
  asm volatile("st.relaxed.cluster.shared::cluster.b32 [%0], %1;" ::"r"(peer_abort), "r"(1) : "memory");
}

__device__ __forceinline__ bool aborted_pair(const PairSmem& sh) {
  return *reinterpret_cast<const volatile int*>(&sh.abort);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    kv_proj_paged_pair_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                              const KvProjParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t ring = smem_u32(smem);  // stage s: A tile at ring + s * kPairStageBytes, B tile after it
  PairSmem& sh = *reinterpret_cast<PairSmem*>(smem + kPairStages * kPairStageBytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_kb = p.k_dim / kBK;
  const uint32_t rank = cluster_ctarank();  // 0: the leader, which issues the MMAs
  const int pair = (int)(blockIdx.x >> 1), pairs = (int)(gridDim.x >> 1);
  // the leader's barriers and the other CTA's abort flag, as cluster addresses
  const uint32_t lead_full = map_to_rank(smem_u32(&sh.full[0]), 0);
  const uint32_t lead_acc_empty = map_to_rank(smem_u32(&sh.acc_empty[0]), 0);
  const uint32_t peer_abort = map_to_rank(smem_u32(&sh.abort), rank ^ 1u);

  if (warp == kMmaWarp) {  // TMEM: the same warp of both CTAs allocates for the pair
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sh.tmem)),
                 "r"(kPairTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&sh.full[s], 1);  // the leader's producer arrives, expecting both CTAs' bytes
      mbar_init(&sh.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.acc_full[b], 1);
      mbar_init(&sh.acc_empty[b], 2 * kEpilogueWarps);
    }
    mbar_init(&sh.mma_done, 1);
    sh.abort = 0;
    sh.issued = sh.consumed = 0;
    fence_barrier_init();
  }
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync_all();  // both CTAs' barriers initialised and the pair's TMEM allocated
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sh.tmem;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      int q = 0;  // k-block loads across this CTA's tiles
      for (int tile = pair; tile < p.tiles && !aborted_pair(sh); tile += pairs) {
        const int n0 = (tile % p.n_tiles) * kPairBN + (int)rank * 128;
        const int m0 = (tile / p.n_tiles) * kPairBM + (int)rank * 128;
        for (int kb = 0; kb < num_kb; ++kb, ++q) {
          const int s = q % kPairStages;
          if (q >= kPairStages && !mbar_wait_bounded(&sh.empty[s], ((q / kPairStages) - 1) & 1)) {
            give_up_pair(sh, peer_abort, p.err);
            break;
          }
          if (aborted_pair(sh)) break;
          const uint32_t bar = lead_full + (uint32_t)(s * 8);
          if (rank == 0) mbar_arrive_expect_tx(&sh.full[s], (uint32_t)(2 * kPairStageBytes));
          const uint32_t a = ring + s * kPairStageBytes;
          tma_load_tile_pair(a, &amap, kb * kBK, m0, bar);
          tma_load_tile_pair(a + kPairTileA, &bmap, kb * kBK, n0, bar);
          *reinterpret_cast<volatile int*>(&sh.issued) = q + 1;
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0 && rank == 0) {
      const uint32_t own_empty = smem_u32(&sh.empty[0]), peer_empty = map_to_rank(own_empty, 1);
      const uint32_t own_acc_full = smem_u32(&sh.acc_full[0]), peer_acc_full = map_to_rank(own_acc_full, 1);
      const uint32_t own_done = smem_u32(&sh.mma_done), peer_done = map_to_rank(own_done, 1);
      int q = 0, i = 0;  // k-blocks consumed, tiles accumulated
      for (int tile = pair; tile < p.tiles && !aborted_pair(sh); tile += pairs, ++i) {
        const int b = i & 1;
        // both CTAs' epilogues must have emptied this accumulator (used two tiles ago)
        if (i >= 2 && !mbar_wait_bounded(&sh.acc_empty[b], ((i >> 1) - 1) & 1)) {
          give_up_pair(sh, peer_abort, p.err);
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + (uint32_t)(b * kPairBN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++q) {
          const int s = q % kPairStages;
          if (!mbar_wait_bounded(&sh.full[s], (q / kPairStages) & 1)) {
            give_up_pair(sh, peer_abort, p.err);
            ok = false;
            break;
          }
          *reinterpret_cast<volatile int*>(&sh.consumed) = q + 1;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a = ring + s * kPairStageBytes, bt = a + kPairTileA;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_bf16_pair(acc, smem_desc(a + k * 32), smem_desc(bt + k * 32), kPairInstrDesc,
                           (kb | k) != 0 ? 1u : 0u);
          umma_commit_pair(own_empty + (uint32_t)(s * 8));  // each CTA's stage is free once read
          umma_commit_pair(peer_empty + (uint32_t)(s * 8));
        }
        if (!ok) break;
        umma_commit_pair(own_acc_full + (uint32_t)(b * 8));  // the tile's accumulators are complete
        umma_commit_pair(peer_acc_full + (uint32_t)(b * 8));
      }
      umma_commit_pair(own_done);  // arrives once every MMA issued above has completed
      umma_commit_pair(peer_done);
    }
  } else {
    // ---- epilogue warps 0-3: TMEM lanes 32w..32w+31 are this CTA's rows 32w..32w+31 of the tile
    int i = 0;
    for (int tile = pair; tile < p.tiles; tile += pairs, ++i) {
      const int b = i & 1;
      // warp-uniform: the tcgen05.ld below needs every lane
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&sh.acc_full[b], (i >> 1) & 1))) {
        give_up_pair(sh, peer_abort, p.err);
        break;
      }
      if (__any_sync(0xffffffffu, aborted_pair(sh))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int n0 = (tile % p.n_tiles) * kPairBN;
      const int64_t t = (int64_t)(tile / p.n_tiles) * kPairBM + (int64_t)rank * 128 + warp * 32 + lane;
      int64_t slot = -1;
      if (t < p.num_tokens) {
        slot = __ldg(p.slots + t);
        if (slot >= p.num_blocks * p.block_size) {
          report(p.err, VFL_DEVERR_SLOT);
          slot = -1;
        }
      }
      const uint32_t acc = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * kPairBN);
      store_rows<kPairBN>(acc, n0, slot, p, lane);
      // this warp has its rows in registers: the accumulator may take the tile after next
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(lead_acc_empty + (uint32_t)(b * 8));
    }
  }

  // ---- teardown. First every thread of both CTAs leaves its loop; then the leader makes every
  // copy either CTA issued land (for a k-block only one CTA loaded, it squares the barrier's
  // count: the arrival the leader never made, or the peer's bytes that never come) and both
  // CTAs wait for the last MMAs; then TMEM is freed.
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync_all();
  if (threadIdx.x == 0) {
    if (!mbar_wait_bounded(&sh.mma_done, 0)) report(p.err, VFL_DEVERR_TIMEOUT);
    if (rank == 0) {
      const int own = *reinterpret_cast<volatile int*>(&sh.issued);
      int other;
      asm volatile("ld.relaxed.cluster.shared::cluster.b32 %0, [%1];"
                   : "=r"(other)
                   : "r"(map_to_rank(smem_u32(&sh.issued), 1))
                   : "memory");
      const int last = own > other ? own : other;
      for (int q = *reinterpret_cast<volatile int*>(&sh.consumed); q < last; ++q) {
        const int s = q % kPairStages;
        if (q >= own) mbar_arrive_expect_tx(&sh.full[s], (uint32_t)kPairStageBytes);  // the peer's copies only
        if (q >= other) mbar_complete_tx(&sh.full[s], (uint32_t)kPairStageBytes);     // the peer's never come
        if (!mbar_wait_bounded(&sh.full[s], (q / kPairStages) & 1)) report(p.err, VFL_DEVERR_TIMEOUT);
      }
    }
  }
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync_all();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPairTmemCols) : "memory");
  }
}

int g_smem_done[2][kMaxDevices];
int g_pair_smem_done[kMaxDevices];

int launch_kv_proj_pair(const void* hidden, int64_t hidden_stride, const void* w_kv, int64_t n, int64_t m_tiles,
                        KvProjParams p, cudaStream_t stream) {
  CUtensorMap amap, bmap;
  int st = make_tensor_map_2d_bf16(hidden, (uint64_t)p.k_dim, (uint64_t)p.num_tokens, (uint64_t)hidden_stride * 2,
                                   kBK, 128, &amap);
  if (st) return st;
  st = make_tensor_map_2d_bf16(w_kv, (uint64_t)p.k_dim, (uint64_t)n, (uint64_t)p.k_dim * 2, kBK, 128, &bmap);
  if (st) return st;
  st = ensure_smem_attribute(reinterpret_cast<const void*>(&kv_proj_paged_pair_kernel), kPairSmemBytes,
                             g_pair_smem_done);
  if (st) return st;
  p.n_tiles = (int32_t)(n / kPairBN);
  p.tiles = (int32_t)(m_tiles * p.n_tiles);
  const int pairs = p.tiles < kNumSMs / 2 ? p.tiles : kNumSMs / 2;  // one persistent pair per two SMs
  kv_proj_paged_pair_kernel<<<2 * pairs, kThreads, kPairSmemBytes, stream>>>(amap, bmap, p);
  return cuda_status(cudaGetLastError(), "kv_proj_paged launch");
}

template <int BN>
int launch_kv_proj(const void* hidden, int64_t hidden_stride, const void* w_kv, int64_t n, int64_t m_tiles,
                   KvProjParams p, cudaStream_t stream) {
  CUtensorMap amap, bmap;
  int st = make_tensor_map_2d_bf16(hidden, (uint64_t)p.k_dim, (uint64_t)p.num_tokens, (uint64_t)hidden_stride * 2,
                                   kBK, kBM, &amap);
  if (st) return st;
  st = make_tensor_map_2d_bf16(w_kv, (uint64_t)p.k_dim, (uint64_t)n, (uint64_t)p.k_dim * 2, kBK, BN, &bmap);
  if (st) return st;
  st = ensure_smem_attribute(reinterpret_cast<const void*>(&kv_proj_paged_kernel<BN>), KvTile<BN>::kSmemBytes,
                             g_smem_done[BN == 256 ? 1 : 0]);
  if (st) return st;
  p.n_tiles = (int32_t)(n / BN);
  p.tiles = (int32_t)(m_tiles * p.n_tiles);
  const int grid = p.tiles < kNumSMs ? p.tiles : kNumSMs;  // one persistent CTA per SM
  kv_proj_paged_kernel<BN><<<grid, kThreads, KvTile<BN>::kSmemBytes, stream>>>(amap, bmap, p);
  return cuda_status(cudaGetLastError(), "kv_proj_paged launch");
}

}  // namespace
}  // namespace vfl

using namespace vfl;

extern "C" int vfl_kv_proj_paged(const void* hidden, int64_t hidden_stride, const void* w_kv, const void* bias,
                                 void* k_cache, void* v_cache, const int64_t* slot_mapping, int64_t num_tokens,
                                 int32_t hidden_dim, int32_t num_heads, int32_t head_dim, int32_t block_size,
                                 int64_t num_blocks, void* stream) {
  if (num_tokens < 0 || num_tokens > (int64_t)1 << 30 || hidden_dim <= 0 || hidden_dim % kBK != 0 ||
      hidden_dim > (1 << 20) || num_heads <= 0 || head_dim <= 0 || head_dim % 32 != 0 || block_size <= 0 ||
      num_blocks <= 0)
    return fail(VFL_ERR_INVALID_ARGUMENT,
                "kv_proj_paged: tokens %lld, hidden_dim %d (a multiple of 64), heads %d, head_dim %d (a multiple "
                "of 32), block_size %d, blocks %lld",
                (long long)num_tokens, hidden_dim, num_heads, head_dim, block_size, (long long)num_blocks);
  const int64_t n = 2LL * num_heads * head_dim;
  if (n % 128 != 0 || n > (1 << 20))
    return fail(VFL_ERR_UNSUPPORTED, "kv_proj_paged: 2 * heads * head_dim = %lld is not a multiple of 128",
                (long long)n);
  if (num_tokens == 0) return VFL_OK;
  if (!hidden || !w_kv || !k_cache || !v_cache || !slot_mapping)
    return fail(VFL_ERR_INVALID_ARGUMENT, "kv_proj_paged: NULL pointer");
  if (!aligned16(hidden) || !aligned16(w_kv) || !aligned16(k_cache) || !aligned16(v_cache) ||
      (hidden_stride * 2) % 16 != 0 || hidden_stride < hidden_dim)
    return fail(VFL_ERR_INVALID_ARGUMENT, "kv_proj_paged: pointers and the hidden row stride must be 16-byte aligned");
  const int64_t m_tiles = (num_tokens + kBM - 1) / kBM;
  if (m_tiles * (n / 128) > INT32_MAX) return fail(VFL_ERR_UNSUPPORTED, "kv_proj_paged: too many tiles");
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
  int st = device_error_word(&p.err);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n % kPairBN == 0 && num_tokens >= kPairMinTokens)
    return launch_kv_proj_pair(hidden, hidden_stride, w_kv, n, (num_tokens + kPairBM - 1) / kPairBM, p, s);
  if (n % 256 == 0) return launch_kv_proj<256>(hidden, hidden_stride, w_kv, n, m_tiles, p, s);
  return launch_kv_proj<128>(hidden, hidden_stride, w_kv, n, m_tiles, p, s);
}
