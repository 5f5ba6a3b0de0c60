// Tensor-core variant of the paged attention kernel: bfloat16, head_dim 64, up to 8 query rows
// of one request per CTA (decode rows, or the beams of a request sharing its encoder pages).
//
// Same work decomposition, producer ring, split-K partials and merge as paged_attention_kernel
// (paged_attention_kernels.cuh); what changes is how a 16-token tile is consumed:
//   * the producer fills the stages with 2-D TMA tensor copies using the 128-byte swizzle, so a
//     tile's 16-byte chunks are spread over all banks (chunk c of row r lands at c ^ (r mod 8));
//   * S[16 tokens x 8 rows] = K_tile . Q^T with mma.m16n8k16 (bf16 in, fp32 accumulate), K as
//     the A operand through ldmatrix, Q held in registers as the B operand;
//   * online softmax on the fp32 accumulators (exp2 domain, lazy rescaling); P is rounded to
//     bf16, staged in shared memory, and O^T[64 x 8] += V^T . P^T with V through ldmatrix.trans.
// One mma.m16n8k16 does 2048 multiply-adds, so a tile costs ~8 mma + ~8 ldmatrix instead of
// ~100 CUDA-core instructions per query row: the beams of a request come almost for free.
// The sum l accumulates the same bf16-rounded p that multiplies V, so the normalisation matches.
#pragma once

#include <cuda.h>

#include "paged_attention_kernels.cuh"

namespace vfl {

constexpr int kTcPTileOffset = 1024;     // P tiles after the SmemHeader
constexpr int kTcRowTableOffset = 2048;  // per-row block-table slices (row_tables plans)
static_assert(sizeof(SmemHeader) <= kTcPTileOffset && kTcPTileOffset + 4 * kTcRows * 16 * 2 <= kTcRowTableOffset &&
                  kTcRowTableOffset + kTcRows * kMaxBlocksPerSplit * 4 <= kTcHeaderBytes,
              "tc header");

// The blocks of one tile position, in a fixed order that the producer and every consumer warp
// derive alike: row j's block unless an earlier row already holds it, with the mask of the rows
// that hold it. Plans without row tables have one block per position, for every row.
struct TileBlocks {
  const int32_t* rows;  // row tables [kTcRows][kMaxBlocksPerSplit], or null
  const int32_t* table; // the request's slice
  int nq;

  __device__ __forceinline__ int count_and_get(int bi, int j, unsigned done, int64_t* phys, unsigned* mask) const {
    // returns the next row >= j that starts a new block (or nq), with that block and its rows
    if (rows == nullptr) {
      if (j > 0) return nq;
      *phys = table[bi];
      *mask = (1u << nq) - 1u;
      return 0;
    }
    while (j < nq && ((done >> j) & 1u)) ++j;
    if (j >= nq) return nq;
    const int32_t b = rows[j * kMaxBlocksPerSplit + bi];
    unsigned m = 0;
    for (int t = j; t < nq; ++t)
      if (rows[t * kMaxBlocksPerSplit + bi] == b) m |= 1u << t;
    *phys = b;
    *mask = m;
    return j;
  }
};

__device__ __forceinline__ uint32_t swz(uint32_t tile_base, int row, int chunk) {
  const uint32_t row_addr = tile_base + row * 128;
  return row_addr + ((chunk ^ ((row_addr >> 7) & 7)) << 4);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16x8x16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2_bits(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}

// A consumer lane's place in the mma fragments and its ldmatrix rows / 16-byte chunks.
struct TcLane {
  int g, tq;                 // mma row group, thread in group
  int k_row, k_chunk_hi;     // K tile rows (A = K through ldmatrix)
  int v_row, v_chunk_hi;     // V tile rows (A = V^T through ldmatrix.trans)
  __device__ __forceinline__ explicit TcLane(int lane) {
    g = lane >> 2;
    tq = lane & 3;
    const int mat = lane >> 3;
    k_row = (lane & 7) + (mat & 1) * 8;
    k_chunk_hi = mat >> 1;
    v_row = (lane & 7) + (mat >> 1) * 8;
    v_chunk_hi = mat & 1;
  }
};

// A consumer warp's running state for its head and this lane's query columns 2tq, 2tq+1:
// max m and sum l per column (exp2 domain), and the O^T m-tiles [dim 16mt + g (+8)][column].
struct TcAccum {
  float m[2], l[2];
  float o[4][4];
  __device__ __forceinline__ void reset() {
    m[0] = m[1] = -INFINITY;
    l[0] = l[1] = 0.f;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mt][e] = 0.f;
  }
  // the l partial sums over the 8 row-group lanes that share each query column
  __device__ __forceinline__ void reduce_l() {
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) l[e] += __shfl_xor_sync(0xffffffffu, l[e], off);
  }
  // column e normalised into the head's 64 outputs at dst (after reduce_l)
  __device__ __forceinline__ void store_output(int e, __nv_bfloat16* dst, const TcLane& ln) const {
    const float inv = l[e] > 0.f ? 1.f / l[e] : 0.f;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      dst[16 * mt + ln.g] = __float2bfloat16_rn(o[mt][e] * inv);
      dst[16 * mt + ln.g + 8] = __float2bfloat16_rn(o[mt][e + 2] * inv);
    }
  }
  // column e's (m, l, acc[64]) partial (after reduce_l)
  __device__ __forceinline__ void store_partial(int e, float* acc, float* ml, const TcLane& ln) const {
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      acc[16 * mt + ln.g] = o[mt][e];
      acc[16 * mt + ln.g + 8] = o[mt][e + 2];
    }
    if (ln.g == 0) *reinterpret_cast<float2*>(ml) = make_float2(m[e], l[e]);
  }
};

// One 16-token tile of one head, in its consumer warp:
//   S[token g, g+8][query 2tq, 2tq+1] = K_tile . Q^T (K through ldmatrix, Q fragments bq);
//   online softmax per query column (exp2 domain, lazy rescaling as in the CUDA-core kernel),
//   masked to the rows the tile's block belongs to (row_on) and to each column's visible tokens;
//   P rounded to bf16 through the warp's shared P tile; O^T += V^T . P^T.
// kt / vt: shared addresses of the head's swizzled K and V tiles. The caller syncs the warp
// before the stage or the P tile is reused.
__device__ __forceinline__ void tc_consume_tile(uint32_t kt, uint32_t vt, const uint32_t (&bq)[4][2],
                                                const bool (&row_on)[2], int tok0, const int (&vis_c)[2],
                                                float scale_log2, __nv_bfloat16* p_tile, uint32_t p_tile_u32,
                                                const TcLane& ln, TcAccum& acc) {
  const int g = ln.g, tq = ln.tq;
  // Every K fragment load first, S in two accumulators (the even and odd 16-dim steps, two mma
  // deep instead of four), and the V fragments, which do not depend on P, loaded before the
  // softmax. (Measured the same as the one-accumulator order: the tile's time is set by the
  // producer's issue rate and the P exchange, not by this chain.)
  uint32_t ka[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) ldsm_x4(swz(kt, ln.k_row, 2 * kk + ln.k_chunk_hi), ka[kk]);
  float sc[4] = {0.f, 0.f, 0.f, 0.f}, sd[4] = {0.f, 0.f, 0.f, 0.f};
  mma_bf16_16x8x16(sc, ka[0], bq[0][0], bq[0][1]);
  mma_bf16_16x8x16(sd, ka[1], bq[1][0], bq[1][1]);
  mma_bf16_16x8x16(sc, ka[2], bq[2][0], bq[2][1]);
  mma_bf16_16x8x16(sd, ka[3], bq[3][0], bq[3][1]);
  uint32_t va[4][4];
#pragma unroll
  for (int mt = 0; mt < 4; ++mt) ldsm_x4_trans(swz(vt, ln.v_row, 2 * mt + ln.v_chunk_hi), va[mt]);
#pragma unroll
  for (int e = 0; e < 4; ++e) sc[e] += sd[e];
  constexpr float kRescaleSlack = 8.f;
  __nv_bfloat16 pb[4];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const bool v0 = row_on[e] && tok0 + g < vis_c[e];
    const bool v1 = row_on[e] && tok0 + g + 8 < vis_c[e];
    const float s0 = v0 ? sc[e] * scale_log2 : -INFINITY;
    const float s1 = v1 ? sc[e + 2] * scale_log2 : -INFINITY;
    float mx = fmaxf(s0, s1);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (mx > acc.m[e] + kRescaleSlack) {
      const float alpha = acc.m[e] == -INFINITY ? 0.f : exp2_approx(acc.m[e] - mx);
      acc.m[e] = mx;
      acc.l[e] *= alpha;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        acc.o[mt][e] *= alpha;
        acc.o[mt][e + 2] *= alpha;
      }
    }
    const bool none = acc.m[e] == -INFINITY;
    pb[e] = __float2bfloat16_rn(none ? 0.f : exp2_approx(s0 - acc.m[e]));
    pb[e + 2] = __float2bfloat16_rn(none ? 0.f : exp2_approx(s1 - acc.m[e]));
    acc.l[e] += __bfloat162float(pb[e]) + __bfloat162float(pb[e + 2]);
  }
  // P -> shared [query][token], then the PV B fragments: query g, tokens 2tq (+1), 2tq+8 (+9)
  p_tile[(2 * tq) * 16 + g] = pb[0];
  p_tile[(2 * tq + 1) * 16 + g] = pb[1];
  p_tile[(2 * tq) * 16 + g + 8] = pb[2];
  p_tile[(2 * tq + 1) * 16 + g + 8] = pb[3];
  __syncwarp();
  uint32_t bp0, bp1;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(bp0) : "r"(p_tile_u32 + (g * 16 + 2 * tq) * 2));
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(bp1) : "r"(p_tile_u32 + (g * 16 + 2 * tq + 8) * 2));
  // O^T += V^T . P^T over the tile's 16 tokens, four 16-dim m-tiles
#pragma unroll
  for (int mt = 0; mt < 4; ++mt) mma_bf16_16x8x16(acc.o[mt], va[mt], bp0, bp1);
}

// The B operand of S = K.Q^T for query row `row` (g < nq) of head h: dims 16kk + 2tq (+1) and
// 16kk + 8 + 2tq (+1); zeros for columns without a row.
__device__ __forceinline__ void tc_load_query(const AttnParams& p, int64_t row, bool on, int h, const TcLane& ln,
                                              uint32_t (&bq)[4][2]) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    bq[kk][0] = bq[kk][1] = 0u;
    if (on) {
      const __nv_bfloat16* src =
          static_cast<const __nv_bfloat16*>(p.q) + row * p.q_stride + h * 64 + kk * 16 + 2 * ln.tq;
      bq[kk][0] = __ldg(reinterpret_cast<const unsigned int*>(src));
      bq[kk][1] = __ldg(reinterpret_cast<const unsigned int*>(src + 8));
    }
  }
}

// Fused KV append, in the consumer warp of head h: the new key and value of each query row
// q0 + j (j < nq) whose new position lies in [pos_lo, pos_hi) go to the row's slot, 16-byte
// pieces (lanes 0-7 the key, 8-15 the value), then a proxy fence orders the stores before the
// producer's TMA (async proxy) reads of the same block. Padding rows (slot < 0) store nothing.
__device__ __forceinline__ void tc_append_rows(const AttnParams& p, int q0, int nq, int q_end, int L, int h,
                                               int pos_lo, int pos_hi, int warp, int lane) {
  using T = __nv_bfloat16;
  constexpr int D = 64;
  const int bs = p.block_size;
  const int64_t capacity = p.num_blocks * (int64_t)bs;
  for (int j = 0; j < nq; ++j) {
    const int t = q0 + j;
    const int pos = p.causal ? L - (q_end - t) : L - 1;
    if (pos < pos_lo || pos >= pos_hi) continue;
    const int64_t slot = __ldg(p.slots + t);
    if (slot < 0) continue;  // padding row
    if (slot >= capacity) {
      if (warp == 0 && lane == 0) report(p.err, VFL_DEVERR_SLOT);
      continue;
    }
    if (lane < 2 * (D / 8)) {
      const int kv = lane >> 3, c = lane & 7;
      const int64_t blk = slot / bs, off = slot - blk * bs;
      const T* src =
          static_cast<const T*>(kv ? p.new_v : p.new_k) + t * (kv ? p.new_v_stride : p.new_k_stride) + h * D + c * 8;
      T* dst = static_cast<T*>(const_cast<void*>(kv ? p.v_cache : p.k_cache)) +
               ((blk * p.num_heads + h) * bs + off) * D + c * 8;
      *reinterpret_cast<uint4*>(dst) = ldg_nc_v4(src);
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  __syncwarp();
}

// kmap / vmap: the K and V pools as 2-D [num_blocks * H * block_size rows, 64 columns] bf16 with
// the 128-byte swizzle; box = 64 columns x (16 * heads_per_cta rows if block_size == 16, else 16).
__global__ void __launch_bounds__(160, 3) paged_attention_tc_kernel(const AttnParams p,
                                                                     const __grid_constant__ CUtensorMap kmap,
                                                                     const __grid_constant__ CUtensorMap vmap) {
  constexpr int D = 64;
  constexpr int TILE = 16 * D;  // elements of one head's 16-token tile (2 KiB)
  using T = __nv_bfloat16;

  extern __shared__ __align__(1024) uint8_t smem[];
  SmemHeader& hdr = *reinterpret_cast<SmemHeader*>(smem);
  T* s_kv = reinterpret_cast<T*>(smem + kTcHeaderBytes);

  const int hpc = p.heads_per_cta;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool producer = warp == hpc;
  const int groups = p.num_heads / hpc;
  const int r = blockIdx.x / groups;
  const int h0 = (blockIdx.x - r * groups) * hpc;
  const int split = blockIdx.y;
  const int bs = p.block_size;
  const int bps = p.blocks_per_split;

  // the item's independent reads in one round trip: the error word, its query range, its length
  // and (producer, one table per request) its split's block-table slice, whatever the length
  // cuts it to - the slice lies inside the table row, and entries past the length go unused
  const unsigned int err_now = load_volatile(p.err);
  const int q_begin = __ldg(p.qsl + r);
  const int q_end = __ldg(p.qsl + r + 1);
  int L = __ldg(p.seq_lens + r);
  int slice_lo = 0, slice_hi = 0;  // entries lane and lane + 32 of the slice
  if (producer && !p.row_tables) {
    const int avail = min(bps, p.table_cols - split * bps);
    const int32_t* src = p.table + (int64_t)r * p.table_stride + (int64_t)split * bps;
    if (lane < avail) slice_lo = __ldg(src + lane);
    if (lane + 32 < avail) slice_hi = __ldg(src + lane + 32);
  }
  if (err_now & VFL_DEVERR_TIMEOUT) return;  // an earlier CTA gave up waiting
  if (bps < 1 || bps > kMaxBlocksPerSplit || p.stages < 2 || p.stages > kMaxStages) {  // the host checks the plan too
    if (threadIdx.x == 0) report(p.err, VFL_DEVERR_CONTEXT);
    return;
  }

  if (q_begin < 0 || q_end < q_begin || q_end > p.total_q) {
    if (threadIdx.x == 0 && split == 0 && blockIdx.z == 0) report(p.err, VFL_DEVERR_QUERY);
    return;
  }
  const int q0 = q_begin + blockIdx.z * kTcRows;
  const int nq = min(kTcRows, q_end - q0);
  if (nq <= 0) return;
  const int cap = min(p.table_cols * bs, p.max_seq_len);
  if (L > cap) {
    if (threadIdx.x == 0 && split == 0 && blockIdx.z == 0) report(p.err, VFL_DEVERR_CONTEXT);
    L = cap;
  }
  L = max(L, 0);
  const int nblk = ceil_div(L, bs);
  const int n_splits = ceil_div(nblk, bps);
  if (split >= max(n_splits, 1)) return;
  // visible tokens of row q0 + j (causal rows see fewer); vis_max bounds the CTA's tiles
  auto visible = [&](int j) { return j < nq ? max(p.causal ? L - (q_end - 1 - (q0 + j)) : L, 0) : 0; };
  const int vis_max = visible(nq - 1) > visible(0) ? visible(nq - 1) : visible(0);
  const int tpb = bs / 16;
  const int blk_begin = split * bps;
  const int tile_begin = blk_begin * tpb;
  const int tile_end = min((blk_begin + bps) * tpb, ceil_div(vis_max, 16));
  const int ntiles = max(0, tile_end - tile_begin);
  const int stages = p.stages;
  const int stage_elems = 2 * hpc * TILE;
  const uint32_t head_tile_bytes = TILE * sizeof(T);

  int32_t* row_tab = reinterpret_cast<int32_t*>(smem + kTcRowTableOffset);
  // fused KV append: each of this CTA's query rows brings one token (the newest position of its
  // sequence; successive positions for causal rows). The split that holds a row's position
  // stores its head group's K and V there - each consumer warp its own head, while the producer
  // already streams the earlier blocks - and the producer waits for those stores before the
  // first unit from the tile of the earliest new position. The block is the row's own (copy-on-
  // write ran before the step), so no other CTA reads these bytes.
  const int new_lo = p.causal ? L - (q_end - q0) : L - 1;   // earliest new position of the rows
  const int new_hi = p.causal ? L - (q_end - (q0 + nq - 1)) : L - 1;
  const int split_lo = blk_begin * bs, split_hi = (blk_begin + bps) * bs;
  const bool appends = p.new_k != nullptr && new_hi >= 0 && new_hi >= split_lo && new_lo < split_hi;
  const int first_new_tile = (new_lo > split_lo ? new_lo : split_lo) / 16;
  if (producer) {
    const int nb = min(bps, nblk - blk_begin);
    const int nrows = p.row_tables ? nq : 1;
    for (int e = lane; e < nrows * nb; e += 32) {
      const int j = e / nb, i = e - j * nb;
      const int64_t trow = p.row_tables ? (int64_t)(q0 + j) : (int64_t)r;
      int b = p.row_tables ? __ldg(p.table + trow * p.table_stride + blk_begin + i) : (e < 32 ? slice_lo : slice_hi);
      if (b < 0 || b >= p.num_blocks) {
        report(p.err, VFL_DEVERR_BLOCK_ID);
        b = 0;
      }
      if (p.row_tables)
        row_tab[j * kMaxBlocksPerSplit + i] = b;
      else
        hdr.table[i] = b;
    }
  }
  const TileBlocks tiles{p.row_tables ? row_tab : nullptr, hdr.table, nq};
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&hdr.full[s], 1);
      mbar_init(&hdr.empty[s], hpc);
    }
    hdr.abort = 0;
    hdr.consumed = 0;
    mbar_init(&hdr.appended, hpc);
    fence_barrier_init();
  }
  __syncthreads();

  if (producer) {
    // units: (tile position, distinct block of the position); u counts them across the item
    int issued = 0;
    if (lane == 0) {
      // One thread issues every copy, so its per-unit bookkeeping is a serial chain that sets
      // how many tiles a CTA keeps in flight: stage, ring round, block and sub-tile advance by
      // counters (no division), and row arithmetic stays in 32 bits.
      const uint64_t policy = p.row_tables ? l2_evict_normal_policy() : l2_evict_first_policy();
      const uint32_t tx_bytes = 2u * hpc * head_tile_bytes;
      const int H = p.num_heads;
      int u = 0, s = 0, round = 0;        // unit u sits in stage s of ring round u / stages
      int blk = blk_begin, sub_tile = 0;  // tile_begin + i == blk * tpb + sub_tile
      bool stop = false, appended = !appends;
      for (int i = 0; i < ntiles && !stop; ++i) {
        const int tile = tile_begin + i;
        if (!appended && tile >= first_new_tile) {  // the consumers' stores of the new K/V first
          appended = true;
          if (!mbar_wait_bounded(&hdr.appended, 0)) {
            report(p.err, VFL_DEVERR_TIMEOUT);
            hdr.abort = 1;
            break;
          }
        }
        unsigned done = 0;
        int64_t phys;
        unsigned mask;
        for (int j = tiles.count_and_get(blk - blk_begin, 0, done, &phys, &mask); j < nq;
             j = tiles.count_and_get(blk - blk_begin, j + 1, done, &phys, &mask)) {
          done |= mask;
          if (round > 0 && !mbar_wait_bounded(&hdr.empty[s], (round - 1) & 1)) {
            report(p.err, VFL_DEVERR_TIMEOUT);
            hdr.abort = 1;
            stop = true;
            break;
          }
          if (*reinterpret_cast<volatile int*>(&hdr.abort)) {
            stop = true;
            break;
          }
          // No proxy fence before the copy: the consumers only read a stage (ldmatrix), those
          // reads have returned before their warp arrives on the stage's empty barrier, and
          // this thread waited on that barrier.
          T* ks = s_kv + s * stage_elems;
          T* vs = ks + hpc * TILE;
          mbar_arrive_expect_tx(&hdr.full[s], tx_bytes);
          // rows of the pool seen as [blocks * H * bs, 64]; the tensor maps bound them to int32
          const int row0 = (static_cast<int>(phys) * H + h0) * bs + sub_tile * 16;
          if (tpb == 1) {  // the head group's tiles are adjacent rows: one box of 16 * hpc rows
            tma_load_2d(ks, &kmap, 0, row0, &hdr.full[s], policy);
            tma_load_2d(vs, &vmap, 0, row0, &hdr.full[s], policy);
          } else {
            for (int w = 0; w < hpc; ++w) {
              tma_load_2d(ks + w * TILE, &kmap, 0, row0 + w * bs, &hdr.full[s], policy);
              tma_load_2d(vs + w * TILE, &vmap, 0, row0 + w * bs, &hdr.full[s], policy);
            }
          }
          issued = ++u;
          if (++s == stages) {
            s = 0;
            ++round;
          }
        }
        if (++sub_tile == tpb) {
          sub_tile = 0;
          ++blk;
        }
      }
      griddep_launch_dependents();  // the combine launch may start; it waits for the grid
    }
    __syncwarp();
    __syncthreads();
    if (lane == 0 && *reinterpret_cast<volatile int*>(&hdr.abort)) {
      for (int t = *reinterpret_cast<volatile int*>(&hdr.consumed); t < issued; ++t)
        mbar_wait_bounded(&hdr.full[t % stages], (t / stages) & 1);
    }
    return;
  }

  // ================= consumers: one warp per head, mma fragments ==========================
  const int h = h0 + warp;
  const TcLane ln(lane);
  const int tq = ln.tq;
  uint32_t bq[4][2];
  tc_load_query(p, q0 + ln.g, ln.g < nq, h, ln, bq);
  if (appends) {  // this warp's head of each row whose new position this split holds
    tc_append_rows(p, q0, nq, q_end, L, h, split_lo, split_hi, warp, lane);
    if (lane == 0) mbar_arrive(&hdr.appended);
  }
  // this thread's two query columns 2tq, 2tq+1
  int vis_c[2];
  vis_c[0] = visible(2 * tq);
  vis_c[1] = visible(2 * tq + 1);
  const bool col_on[2] = {2 * tq < nq, 2 * tq + 1 < nq};
  TcAccum acc;
  acc.reset();
  // this warp's P tile: [8 query rows][16 tokens] bf16
  T* p_tile = reinterpret_cast<T*>(smem + kTcPTileOffset) + warp * (kTcRows * 16);
  const uint32_t p_tile_u32 = smem_u32(p_tile);

  bool aborted = false;
  // unit u sits in stage s of ring round u / stages; tile_begin + i == (blk_begin + bi) * tpb + sub
  int u = 0, s = 0, round = 0, bi = 0, sub = 0;
  const uint32_t kt0 = smem_u32(s_kv + warp * TILE);
  const uint32_t stage_bytes = stage_elems * sizeof(T);
  const uint32_t v_off = hpc * TILE * sizeof(T);
#pragma unroll 1
  for (int i = 0; i < ntiles && !aborted; ++i) {
    const int tok0 = (tile_begin + i) * 16;
    unsigned done = 0;
    int64_t phys_unused;
    unsigned mask;
#pragma unroll 1
    for (int j = tiles.count_and_get(bi, 0, done, &phys_unused, &mask); j < nq;
         j = tiles.count_and_get(bi, j + 1, done, &phys_unused, &mask)) {
      done |= mask;
      if (!mbar_wait_bounded(&hdr.full[s], round & 1)) {
        report(p.err, VFL_DEVERR_TIMEOUT);
        if (lane == 0) {
          hdr.abort = 1;
          atomicMax(&hdr.consumed, u);
        }
        aborted = true;
        break;
      }
      const uint32_t kt = kt0 + s * stage_bytes;
      // the rows this unit's block belongs to (every row without row tables)
      const bool row_on[2] = {col_on[0] && ((mask >> (2 * tq)) & 1u), col_on[1] && ((mask >> (2 * tq + 1)) & 1u)};
      tc_consume_tile(kt, kt + v_off, bq, row_on, tok0, vis_c, p.scale_log2, p_tile, p_tile_u32, ln, acc);
      __syncwarp();  // P tile and K/V stage reads done before the next tile reuses them
      if (lane == 0) mbar_arrive(&hdr.empty[s]);
      ++u;
      if (++s == stages) {
        s = 0;
        ++round;
      }
    }
    if (++sub == tpb) {
      sub = 0;
      ++bi;
    }
  }
  __syncthreads();
  if (aborted || *reinterpret_cast<volatile int*>(&hdr.abort)) return;
  acc.reduce_l();

  const int S = p.num_splits;
  if (n_splits <= 1) {
#pragma unroll
    for (int e = 0; e < 2; ++e)
      if (col_on[e])
        acc.store_output(e, static_cast<T*>(p.out) + (int64_t)(q0 + 2 * tq + e) * p.out_stride + h * D, ln);
    return;
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    if (!col_on[e]) continue;
    const int64_t item = ((int64_t)(q0 + 2 * tq + e) * p.num_heads + h) * S + split;
    acc.store_partial(e, p.ws_acc + item * D, p.ws_ml + item * 2, ln);
  }
  if (p.ws_arrivals == nullptr) return;  // the combine launch merges
  consumer_barrier(hpc);
  if (threadIdx.x == 0) {
    int* arrivals = p.ws_arrivals + ((int64_t)r * groups + h0 / hpc) * gridDim.z + blockIdx.z;
    hdr.is_last = arrive_acq_rel(arrivals) == n_splits - 1;
  }
  consumer_barrier(hpc);
  if (!hdr.is_last) return;
  for (int j = 0; j < nq; ++j) merge_splits<T, D>(p, q0 + j, h, n_splits, lane);
}

}  // namespace vfl
