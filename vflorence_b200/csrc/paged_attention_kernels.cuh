// Paged decode / cross attention for B200 (sm_100a).
//
// Work item (one CTA): request r, a group of `heads_per_cta` adjacent heads (one warp each), one
// split-K range of the request's KV blocks, and up to QPC query rows of the request (QPC = 1
// for decoder self-attention; 4 for rows that share a request's pages, e.g. beams over one
// encoder output - those rows read every K/V page once).
//
// Data path: the pool layout [num_blocks, H, block_size, D] makes a (block, head-group) 16-token
// K tile one contiguous chunk, so one elected thread streams tiles into a ring of shared-memory
// stages with cp.async.bulk (TMA bulk copies completing on mbarriers); warps consume them with
// 16-byte shared loads. No tensor cores: one query row per head is ~1 flop per byte.
//
// Per 16-token tile and head, in a warp:
//   QK: lanes = (token-in-pass `tip`, 16-element slice `sub`); q slice lives in registers,
//       pre-scaled by scale*log2(e); partial dots are reduced over the slice lanes by xor shuffles.
//   online softmax in the exp2 domain (running max m, running sum l).
//   PV: lanes = (16-byte V chunk `dch`, token subgroup `tsub`); p is fetched from the QK lanes by
//       shuffle; per-lane fp32 accumulators are reduced over `tsub` once per work item.
// A work item whose request needs one split writes the normalised output; otherwise it writes
// (m, l, acc) partials, merged either by the last split CTA of the (request, head group) to
// finish - counted on an arrival counter that the launcher clears; chosen for latency-bound
// calls - or by a separate combine launch (bandwidth-bound calls, where waiting on the counter
// would hold every split CTA's SM slot).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace vfl {

struct AttnParams {
  const void* q;
  int64_t q_stride;  // elements between query rows
  const void* k_cache;
  const void* v_cache;
  int64_t num_blocks;
  void* out;
  int64_t out_stride;
  const int32_t* qsl;       // [num_reqs + 1]
  const int32_t* seq_lens;  // [num_reqs]
  const int32_t* table;     // [num_reqs, table_stride], or [total_q, table_stride] with row_tables
  int64_t table_stride;
  int32_t table_cols;
  int32_t num_reqs;
  int32_t total_q;
  int32_t num_heads;
  int32_t block_size;
  int32_t causal;
  int32_t heads_per_cta;
  int32_t blocks_per_split;
  int32_t num_splits;  // workspace stride (max splits of any request)
  int32_t stages;
  int32_t max_seq_len;  // planned maximum; longer device lengths are clamped and reported
  int32_t row_tables;   // 1: one block table per query row (tensor-core kernel only)
  int32_t schedule;     // VFL_SCHEDULE_ITEMS or VFL_SCHEDULE_BALANCED (tensor-core kernel only)
  int32_t min_tiles;    // balanced: fewest 16-token tiles a CTA takes
  int32_t balanced_ctas;  // balanced: CTAs of the grid (partial records in the workspace)
  int32_t max_q_len;      // balanced: most query rows of a request (rows of the merge grid)
  float scale_log2;  // softmax scale * log2(e)
  float* ws_acc;     // [total_q, H, num_splits, D]
  float* ws_ml;      // [total_q, H, num_splits, 2]
  int* ws_arrivals;  // [num_reqs, H / heads_per_cta, q_chunks], zero at launch; null: the
                     // combine kernel merges the partials instead
  int4* ws_desc;     // balanced: [num_reqs, H / heads_per_cta] where each item's pieces went
  // fused KV append (null: the caches already hold every token): query row t's new key / value,
  // [H, D] dense at new_k + t * new_k_stride, go to slot slots[t] (< 0: none) before the item
  // reads the block that holds them
  const void* new_k;
  const void* new_v;
  int64_t new_k_stride;
  int64_t new_v_stride;
  const int64_t* slots;
  unsigned int* err;
};

constexpr int kMaxBlocksPerSplit = 64;
constexpr int kMaxStages = 8;
constexpr int kHeaderBytes = 1024;  // block-table slice, full/empty barriers, flags
constexpr int kMaxStageBytes = 64 * 1024;

// Shared-memory header layout.
struct SmemHeader {
  int32_t table[kMaxBlocksPerSplit];  // this item's block ids (validated)
  uint64_t full[kMaxStages];          // stage s holds tile data (TMA transaction bytes)
  uint64_t empty[kMaxStages];         // every consumer warp is done with stage s
  int abort;                          // a bounded wait gave up
  int consumed;                       // tiles consumed before an abort
  int is_last;                        // this CTA is the last split of its item to finish
  uint64_t appended;                  // fused KV append: every consumer warp stored its head's
                                      // new K/V
};
static_assert(sizeof(SmemHeader) <= kHeaderBytes, "header");

// Merges the split-K partials of one (query row, head) into the output: one warp, lane s holds
// the weight of split s (32 at a time) and broadcasts it; each lane owns D/32 dims. Partials are
// read through L2 (other CTAs wrote them).
template <typename T, int D>
__device__ __forceinline__ void merge_splits(const AttnParams& p, int row, int h, int n_splits, int lane) {
  constexpr int DPL = (D + 31) / 32;
  const int64_t item0 = ((int64_t)row * p.num_heads + h) * p.num_splits;
  const float2* ml = reinterpret_cast<const float2*>(p.ws_ml) + item0;
  float M = -INFINITY;
  for (int s = lane; s < n_splits; s += 32) M = fmaxf(M, __ldcg(ml + s).x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float* acc = p.ws_acc + item0 * D;
  float a[DPL];
#pragma unroll
  for (int k = 0; k < DPL; ++k) a[k] = 0.f;
  float Lsum = 0.f;
  if (M != -INFINITY) {
    for (int s0 = 0; s0 < n_splits; s0 += 32) {
      float w = 0.f;
      if (s0 + lane < n_splits) {
        const float2 v = __ldcg(ml + s0 + lane);
        w = exp2f(v.x - M);
        Lsum = fmaf(w, v.y, Lsum);
      }
      const int n = min(32, n_splits - s0);
#pragma unroll 4
      for (int j = 0; j < n; ++j) {
        const float wj = __shfl_sync(0xffffffffu, w, j);
        const float* src = acc + (int64_t)(s0 + j) * D;
#pragma unroll
        for (int k = 0; k < DPL; ++k)
          if (lane + 32 * k < D) a[k] = fmaf(wj, __ldcg(src + lane + 32 * k), a[k]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) Lsum += __shfl_xor_sync(0xffffffffu, Lsum, o);
  const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
  T* out = static_cast<T*>(p.out) + (int64_t)row * p.out_stride + h * D;
#pragma unroll
  for (int k = 0; k < DPL; ++k) {
    const int d = lane + 32 * k;
    if (d >= D) continue;
    const float v = a[k] * inv;
    if constexpr (sizeof(T) == 4) {
      out[d] = v;
    } else {
      out[d] = __float2bfloat16_rn(v);
    }
  }
}

// atomicAdd(1) with acquire-release semantics at GPU scope; returns the previous count.
__device__ __forceinline__ int arrive_acq_rel(int* counter) {
  int prev;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(prev) : "l"(counter) : "memory");
  return prev;
}

__device__ __forceinline__ void consumer_barrier(int consumers) {
  asm volatile("bar.sync 1, %0;" ::"r"(consumers * 32) : "memory");
}

// Warp roles: warps [0, heads_per_cta) consume (one head each); warp heads_per_cta produces.
template <typename T, int D, int QPC>
__global__ void __launch_bounds__(160, QPC == 1 ? 3 : 2) paged_attention_kernel(const AttnParams p) {
  constexpr int VEC = Elem<T>::kVec;         // elements per 16-byte vector
  constexpr int NCH = 16 / VEC;              // 16-byte chunks in a lane's 16-element QK slice
  constexpr int TPT_RAW = D / 16;            // slice lanes that hold data
  constexpr int TPT = next_pow2(TPT_RAW);    // lanes per token in QK
  constexpr int TPP = 32 / TPT;              // tokens per QK pass
  constexpr int PASSES = 16 / TPP;           // QK passes per 16-token tile
  constexpr int DCH = D / VEC;               // 16-byte chunks per K/V row
  constexpr int DCHP = next_pow2(DCH);
  constexpr int TSUB = DCHP >= 32 ? 1 : 32 / DCHP;  // token subgroups in PV
  constexpr int CPL = DCHP >= 32 ? DCHP / 32 : 1;   // V chunks per lane in PV
  constexpr int TOKPV = 16 / TSUB;                  // tokens per lane per tile in PV
  constexpr int TILE = 16 * D;                      // elements of one head's 16-token tile
  static_assert(D % 16 == 0 && TPT <= 32 && TPP <= 16, "head_dim");
  static_assert(TPP % TSUB == 0, "PV token subgroups must nest in QK passes");

  extern __shared__ __align__(128) uint8_t smem[];
  SmemHeader& hdr = *reinterpret_cast<SmemHeader*>(smem);
  T* s_kv = reinterpret_cast<T*>(smem + kHeaderBytes);

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
  // and (producer) its split's block-table slice, whatever the length cuts it to - the slice
  // lies inside the table row, and entries past the length go unused
  const unsigned int err_now = load_volatile(p.err);
  const int q_begin = __ldg(p.qsl + r);
  const int q_end = __ldg(p.qsl + r + 1);
  int L = __ldg(p.seq_lens + r);
  int slice_lo = 0, slice_hi = 0;  // entries lane and lane + 32 of the slice
  if (producer) {
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

  // ---- this CTA's query rows and visible lengths (uniform across the CTA)
  if (q_begin < 0 || q_end < q_begin || q_end > p.total_q) {
    if (threadIdx.x == 0 && split == 0 && blockIdx.z == 0) report(p.err, VFL_DEVERR_QUERY);
    return;
  }
  const int q0 = q_begin + blockIdx.z * QPC;
  const int nq = min(QPC, q_end - q0);
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

  int vis[QPC];
  int vis_max = 0, vis_min = 0x7fffffff;
#pragma unroll
  for (int j = 0; j < QPC; ++j) {
    const int row = q0 + j;
    int v = 0;
    if (j < nq) v = p.causal ? L - (q_end - 1 - row) : L;
    v = max(v, 0);
    vis[j] = v;
    vis_max = max(vis_max, v);
    if (j < nq) vis_min = min(vis_min, v);
  }
  const int tpb = bs / 16;  // 16-token tiles per block
  const int blk_begin = split * bps;
  const int tile_begin = blk_begin * tpb;
  const int tile_end = min((blk_begin + bps) * tpb, ceil_div(vis_max, 16));
  const int ntiles = max(0, tile_end - tile_begin);
  const int stages = p.stages;
  const int stage_elems = 2 * hpc * TILE;
  const uint32_t head_tile_bytes = TILE * sizeof(T);
  // fused KV append (one query row per request; the host admits no other plan): the row's new
  // token is its sequence's newest position L - 1. The split that holds it stores the head
  // group's K and V there - each consumer warp its own head, while the producer already streams
  // the earlier tiles - and the producer waits for those stores before the tile that holds the
  // position. The block is the row's own (copy-on-write ran before the step).
  const int new_pos = L - 1;
  const bool appends = QPC == 1 && p.new_k != nullptr && nq == 1 && new_pos >= blk_begin * bs &&
                       new_pos < (blk_begin + bps) * bs;
  const int new_tile = new_pos / 16;

  // ---- set-up: the producer stages the block-table slice, thread 0 the barriers
  if (producer) {
    const int nb = min(bps, nblk - blk_begin);
    for (int i = lane; i < nb; i += 32) {
      int b = i < 32 ? slice_lo : slice_hi;
      if (b < 0 || b >= p.num_blocks) {
        report(p.err, VFL_DEVERR_BLOCK_ID);
        b = 0;  // read a valid block instead; the error word flags the result as garbage
      }
      hdr.table[i] = b;
    }
  }
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
    // ================= producer: stream tiles into the stage ring ==========================
    int issued = 0;
    if (lane == 0) {
      const uint64_t policy = l2_evict_first_policy();
      bool appended = !appends;
      // tile i sits in stage s of ring round i / stages, tile_begin + i == blk * tpb + sub_tile:
      // counters, not divisions, on this thread's per-tile chain
      int s = 0, round = 0, blk = blk_begin, sub_tile = 0;
      for (int i = 0; i < ntiles; ++i) {
        if (!appended && tile_begin + i >= new_tile) {  // the consumers' stores of the new K/V first
          appended = true;
          if (!mbar_wait_bounded(&hdr.appended, 0)) {
            report(p.err, VFL_DEVERR_TIMEOUT);
            hdr.abort = 1;
            break;
          }
        }
        if (round > 0 && !mbar_wait_bounded(&hdr.empty[s], (round - 1) & 1)) {
          report(p.err, VFL_DEVERR_TIMEOUT);
          hdr.abort = 1;
          break;
        }
        if (*reinterpret_cast<volatile int*>(&hdr.abort)) break;
        // no proxy fence before the copy: the consumers only read a stage, and their reads
        // have returned before they arrive on its empty barrier, which this thread waited on
        const int64_t phys = hdr.table[blk - blk_begin];
        T* ks = s_kv + s * stage_elems;
        T* vs = ks + hpc * TILE;
        mbar_arrive_expect_tx(&hdr.full[s], 2u * hpc * head_tile_bytes);
        const int64_t base = ((phys * p.num_heads + h0) * bs + sub_tile * 16) * D;
        if (tpb == 1) {  // the head group's tiles are adjacent: one copy each for K and V
          bulk_copy_g2s_hint(ks, static_cast<const T*>(p.k_cache) + base, hpc * head_tile_bytes,
                             &hdr.full[s], policy);
          bulk_copy_g2s_hint(vs, static_cast<const T*>(p.v_cache) + base, hpc * head_tile_bytes,
                             &hdr.full[s], policy);
        } else {
          for (int w = 0; w < hpc; ++w) {
            const int64_t off = base + (int64_t)w * bs * D;
            bulk_copy_g2s_hint(ks + w * TILE, static_cast<const T*>(p.k_cache) + off, head_tile_bytes,
                               &hdr.full[s], policy);
            bulk_copy_g2s_hint(vs + w * TILE, static_cast<const T*>(p.v_cache) + off, head_tile_bytes,
                               &hdr.full[s], policy);
          }
        }
        issued = i + 1;
        if (++s == stages) {
          s = 0;
          ++round;
        }
        if (++sub_tile == tpb) {
          sub_tile = 0;
          ++blk;
        }
      }
      griddep_launch_dependents();  // the combine launch may start; it waits for the grid
    }
    __syncwarp();
    __syncthreads();  // pairs with the consumers' barrier below
    if (lane == 0 && *reinterpret_cast<volatile int*>(&hdr.abort)) {
      // Let copies still in flight land (bounded) before the CTA's shared memory is released.
      for (int t = *reinterpret_cast<volatile int*>(&hdr.consumed); t < issued; ++t)
        mbar_wait_bounded(&hdr.full[t % stages], (t / stages) & 1);
    }
    return;
  }

  // ================= consumers: one warp per head ==========================================
  const int h = h0 + warp;
  // query slice in registers: chunk c of the registers pairs with shared chunk (c+rot)%NCH
  const int sub = lane % TPT;
  const int tip = lane / TPT;
  const bool qk_on = sub < TPT_RAW;
  const int rot = (((lane & 7) * NCH) >> 3) % NCH;  // spreads a quarter-warp over all banks
  float qr[QPC][16];
#pragma unroll
  for (int j = 0; j < QPC; ++j) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      float f[VEC];
      if (j < nq && qk_on) {
        const int cc = (c + rot) % NCH;
        const T* src = static_cast<const T*>(p.q) + (int64_t)(q0 + j) * p.q_stride + h * D +
                       sub * 16 + cc * VEC;
        unpack16(ldg_nc_v4(src), f, T());
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) f[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) qr[j][c * VEC + e] = f[e] * p.scale_log2;
    }
  }
  if (appends) {  // this warp's head of the row's new token, in 16-byte pieces
    const int t = q0;
    const int64_t slot = __ldg(p.slots + t);
    const int64_t capacity = p.num_blocks * (int64_t)bs;
    if (slot >= capacity) {
      if (warp == 0 && lane == 0) report(p.err, VFL_DEVERR_SLOT);
    } else if (slot >= 0) {  // slot < 0: a padding row, nothing to store
      const int64_t blk = slot / bs, off = slot - blk * bs;
      for (int c = lane; c < 2 * DCH; c += 32) {
        const int kv = c >= DCH, ch = kv ? c - DCH : c;
        const T* src = static_cast<const T*>(kv ? p.new_v : p.new_k) + t * (kv ? p.new_v_stride : p.new_k_stride) +
                       h * D + ch * VEC;
        T* dst = static_cast<T*>(const_cast<void*>(kv ? p.v_cache : p.k_cache)) +
                 ((blk * p.num_heads + h) * bs + off) * D + ch * VEC;
        *reinterpret_cast<uint4*>(dst) = ldg_nc_v4(src);
      }
    }
    // the stores above, before the producer's bulk (async proxy) copies of the same block
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&hdr.appended);
  }
  int koff[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) koff[c] = sub * 16 + ((c + rot) % NCH) * VEC;

  const int dch = DCHP >= 32 ? lane : lane % DCHP;
  const int tsub = DCHP >= 32 ? 0 : lane / DCHP;
  bool pv_on[CPL];
#pragma unroll
  for (int c = 0; c < CPL; ++c) pv_on[c] = dch + 32 * c < DCH;

  float m[QPC], l[QPC], acc[QPC][CPL * VEC];
#pragma unroll
  for (int j = 0; j < QPC; ++j) {
    m[j] = -INFINITY;
    l[j] = 0.f;
#pragma unroll
    for (int e = 0; e < CPL * VEC; ++e) acc[j][e] = 0.f;
  }

  bool aborted = false;
  int s = 0, round = 0;  // tile i sits in stage s of ring round i / stages
#pragma unroll 1
  for (int i = 0; i < ntiles; ++i) {
    if (!mbar_wait_bounded(&hdr.full[s], round & 1)) {
      report(p.err, VFL_DEVERR_TIMEOUT);
      if (lane == 0) {
        hdr.abort = 1;
        atomicMax(&hdr.consumed, i);
      }
      aborted = true;
      break;
    }
    const T* kt = s_kv + (size_t)s * stage_elems + warp * TILE;
    const T* vt = kt + hpc * TILE;
    const int tok0 = (tile_begin + i) * 16;
    const bool full = tok0 + 16 <= vis_min;

    // QK
    float sc[QPC][PASSES];
#pragma unroll
    for (int ps = 0; ps < PASSES; ++ps) {
      const int t = ps * TPP + tip;
      float kf[16];
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (qk_on) v = *reinterpret_cast<const uint4*>(kt + t * D + koff[c]);
        unpack16(v, kf + c * VEC, T());
      }
#pragma unroll
      for (int j = 0; j < QPC; ++j) {
        float d0 = 0.f, d1 = 0.f;
#pragma unroll
        for (int e = 0; e < 16; e += 2) fma2(d0, d1, qr[j][e], qr[j][e + 1], kf[e], kf[e + 1]);
        float dot = d0 + d1;
#pragma unroll
        for (int o = 1; o < TPT; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        sc[j][ps] = (full || tok0 + t < vis[j]) ? dot : -INFINITY;
      }
    }
    // online softmax in the exp2 domain. The running reference m only moves when the tile's
    // maximum exceeds it by more than kRescaleSlack (so p = 2^(s - m) <= 2^kRescaleSlack stays
    // far from overflow); acc and l always share that reference, so the result is unchanged.
    constexpr float kRescaleSlack = 8.f;
#pragma unroll
    for (int j = 0; j < QPC; ++j) {
      float mx = sc[j][0];
#pragma unroll
      for (int ps = 1; ps < PASSES; ++ps) mx = fmaxf(mx, sc[j][ps]);
#pragma unroll
      for (int o = TPT; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (mx > m[j] + kRescaleSlack) {  // warp-uniform
        const float alpha = m[j] == -INFINITY ? 0.f : exp2_approx(m[j] - mx);
        m[j] = mx;
        l[j] *= alpha;
#pragma unroll
        for (int e = 0; e < CPL * VEC; ++e) acc[j][e] *= alpha;
      }
      const bool none = m[j] == -INFINITY;  // nothing visible yet for this row
#pragma unroll
      for (int ps = 0; ps < PASSES; ++ps) sc[j][ps] = none ? 0.f : exp2_approx(sc[j][ps] - m[j]);
    }
    // PV
#pragma unroll
    for (int k = 0; k < TOKPV; ++k) {
      const int ps = (TSUB * k) / TPP;  // compile-time: tsub < TSUB and TSUB divides TPP
      const int t = tsub + TSUB * k;
      const int src = (t - ps * TPP) * TPT;
      float vf[CPL * VEC];
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (pv_on[c]) v = *reinterpret_cast<const uint4*>(vt + t * D + (dch + 32 * c) * VEC);
        unpack16(v, vf + c * VEC, T());
      }
#pragma unroll
      for (int j = 0; j < QPC; ++j) {
        const float pj = __shfl_sync(0xffffffffu, sc[j][ps], src);
        if (full || tok0 + t < vis[j]) {  // masked tokens may hold anything, even NaN
          l[j] += pj;
#pragma unroll
          for (int e = 0; e < CPL * VEC; e += 2) fma2(acc[j][e], acc[j][e + 1], pj, pj, vf[e], vf[e + 1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&hdr.empty[s]);  // this warp is done with stage s
    if (++s == stages) {
      s = 0;
      ++round;
    }
  }
  __syncthreads();  // pairs with the producer's barrier (abort bookkeeping)
  if (aborted || *reinterpret_cast<volatile int*>(&hdr.abort)) return;

  // ---- reduce the PV accumulators over token subgroups
#pragma unroll
  for (int o = DCHP; o < 32; o <<= 1) {
#pragma unroll
    for (int j = 0; j < QPC; ++j) {
      l[j] += __shfl_xor_sync(0xffffffffu, l[j], o);
#pragma unroll
      for (int e = 0; e < CPL * VEC; ++e) acc[j][e] += __shfl_xor_sync(0xffffffffu, acc[j][e], o);
    }
  }
  const int S = p.num_splits;
  if (n_splits <= 1) {  // the whole request in this CTA: normalise and store
    if (tsub != 0) return;
#pragma unroll
    for (int j = 0; j < QPC; ++j) {
      if (j >= nq) break;
      const int row = q0 + j;
      const float inv = l[j] > 0.f ? 1.f / l[j] : 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        if (!pv_on[c]) continue;
        float f[VEC];
#pragma unroll
        for (int e = 0; e < VEC; ++e) f[e] = acc[j][c * VEC + e] * inv;
        T* dst = static_cast<T*>(p.out) + (int64_t)row * p.out_stride + h * D + (dch + 32 * c) * VEC;
        *reinterpret_cast<uint4*>(dst) = pack16(f, T());
      }
    }
    return;
  }
  // split request: store this split's (m, l, acc) partials ...
  if (tsub == 0) {
#pragma unroll
    for (int j = 0; j < QPC; ++j) {
      if (j >= nq) break;
      const int64_t item = ((int64_t)(q0 + j) * p.num_heads + h) * S + split;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        if (!pv_on[c]) continue;
        float4* dst = reinterpret_cast<float4*>(p.ws_acc + item * D + (dch + 32 * c) * VEC);
#pragma unroll
        for (int e = 0; e < VEC; e += 4)
          dst[e / 4] = make_float4(acc[j][c * VEC + e], acc[j][c * VEC + e + 1],
                                   acc[j][c * VEC + e + 2], acc[j][c * VEC + e + 3]);
      }
      if (lane == 0) *reinterpret_cast<float2*>(p.ws_ml + item * 2) = make_float2(m[j], l[j]);
    }
  }
  if (p.ws_arrivals == nullptr) return;  // the combine launch merges
  // ... and the last split of (request, head group, query chunk) to arrive merges them all:
  // CTA barrier, then one thread publishes the CTA's writes (release) with its arrival; the
  // last arriver acquires everyone's partials before the CTA barrier that releases its warps.
  consumer_barrier(hpc);
  if (threadIdx.x == 0) {
    int* arrivals = p.ws_arrivals + ((int64_t)r * groups + h0 / hpc) * gridDim.z + blockIdx.z;
    hdr.is_last = arrive_acq_rel(arrivals) == n_splits - 1;
  }
  consumer_barrier(hpc);
  if (!hdr.is_last) return;
  for (int j = 0; j < nq && j < QPC; ++j) merge_splits<T, D>(p, q0 + j, h, n_splits, lane);
}

// Separate merge launch: one warp per (query row, head) of a request that was split.
template <typename T, int D>
__global__ void __launch_bounds__(128) paged_attention_combine_kernel(const AttnParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= (int64_t)p.total_q * p.num_heads) return;
  const int row = static_cast<int>(gw / p.num_heads);
  const int h = static_cast<int>(gw - (int64_t)row * p.num_heads);
  int lo = 0, hi = p.num_reqs - 1;  // request owning this row: last r with qsl[r] <= row
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(p.qsl + mid) <= row) lo = mid; else hi = mid - 1;
  }
  if (row < __ldg(p.qsl + lo) || row >= __ldg(p.qsl + lo + 1)) return;  // row of no request
  int L = min(__ldg(p.seq_lens + lo), min(p.table_cols * p.block_size, p.max_seq_len));
  L = max(L, 0);
  const int n_splits = ceil_div(ceil_div(L, p.block_size), p.blocks_per_split);
  if (n_splits <= 1) return;  // written directly by the main kernel
  griddep_wait();             // launched as the attention grid's programmatic dependent
  merge_splits<T, D>(p, row, h, n_splits, lane);
}

// Launches `kernel` as the programmatic dependent of the grid launched before it on `stream`:
// its CTAs may start while that grid drains, and wait for it with griddepcontrol.wait.
template <typename... Params, typename... Args>
int launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, cudaStream_t stream, const char* what,
                     Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, args...), what);
}

// Tensor-core variant (paged_attention_tc.cuh): bf16, head_dim 64, up to kTcRows rows per CTA.
constexpr int kTcHeaderBytes = 4096;  // SmemHeader | one 8x16 bf16 P tile per consumer warp | row tables
constexpr int kTcRows = 8;            // query rows per CTA (the mma N dimension)

// Balanced schedule (paged_attention_balanced.cuh).
constexpr int kBalancedMaxReqs = 2048;  // requests whose lengths and rows fit in shared memory
constexpr int kBalancedMaxLen = 1 << 24;  // tokens per request: the int32 tile prefix of 2048
                                          // requests stays below 2^31 (and lengths pack with
                                          // the row count into 32 bits)
constexpr int kBalancedCtasPerSM = 3;   // the kernel's launch bounds (registers)
constexpr int kBalancedMinTiles = 8;    // default fewest 16-token tiles per CTA

// Shared-memory bytes of its per-request arrays: tile prefix [R + 1], packed length and rows
// [R], first query row [R].
inline __host__ __device__ int balanced_sched_bytes(int num_reqs) {
  return ((3 * num_reqs + 1) * 4 + 15) / 16 * 16;
}

// Its workspace: partial records acc [ctas, 2, hpc, kTcRows, 64] f32 | (m, l) [.., 2] f32 |
// item directory [num_reqs, H / hpc] int4; each part 256-byte aligned.
struct BalancedWorkspace {
  int64_t acc_bytes, ml_bytes, desc_bytes;
  __host__ __device__ BalancedWorkspace(int64_t ctas, int hpc, int64_t num_reqs, int num_heads) {
    const int64_t recs = ctas * 2 * hpc * kTcRows;
    acc_bytes = (recs * 64 * 4 + 255) / 256 * 256;
    ml_bytes = (recs * 2 * 4 + 255) / 256 * 256;
    desc_bytes = (num_reqs * (num_heads / hpc) * 16 + 255) / 256 * 256;
  }
  __host__ __device__ int64_t total() const { return acc_bytes + ml_bytes + desc_bytes; }
};
int launch_paged_attention_tc(const AttnParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap, dim3 grid,
                              int threads, int smem_bytes, cudaStream_t stream);

// Launches the kernel; defined per dtype.
int launch_paged_attention_f32(const AttnParams& p, int head_dim, int qpc, dim3 grid, int threads,
                               int smem_bytes, cudaStream_t stream);
int launch_paged_attention_bf16(const AttnParams& p, int head_dim, int qpc, dim3 grid, int threads,
                                int smem_bytes, cudaStream_t stream);

template <typename T, int D, int QPC>
int launch_one(const AttnParams& p, dim3 grid, int threads, int smem_bytes, cudaStream_t stream) {
  static int smem_done[kMaxDevices];
  auto kernel = paged_attention_kernel<T, D, QPC>;
  // the ring of most plans fits kMaxStageBytes; head_dim 512 needs two stages of up to 64 KiB
  const int want = smem_bytes > kHeaderBytes + kMaxStageBytes ? smem_bytes : kHeaderBytes + kMaxStageBytes;
  int st = ensure_smem_attribute(reinterpret_cast<const void*>(kernel), want, smem_done);
  if (st) return st;
  kernel<<<grid, threads, smem_bytes, stream>>>(p);
  st = cuda_status(cudaGetLastError(), "paged_attention launch");
  if (st || p.num_splits <= 1 || p.ws_arrivals != nullptr) return st;
  const int64_t warps = (int64_t)p.total_q * p.num_heads;
  return launch_dependent(paged_attention_combine_kernel<T, D>, dim3(static_cast<unsigned>(ceil_div(warps, (int64_t)4))),
                          dim3(128), stream, "paged_attention combine launch", p);
}

template <typename T, int D>
int launch_qpc(const AttnParams& p, int qpc, dim3 grid, int threads, int smem_bytes, cudaStream_t stream) {
  if (qpc == 1) return launch_one<T, D, 1>(p, grid, threads, smem_bytes, stream);
  return launch_one<T, D, 4>(p, grid, threads, smem_bytes, stream);
}

template <typename T>
int launch_dtype(const AttnParams& p, int head_dim, int qpc, dim3 grid, int threads, int smem_bytes,
                 cudaStream_t stream) {
  switch (head_dim) {
    case 32: return launch_qpc<T, 32>(p, qpc, grid, threads, smem_bytes, stream);
    case 48: return launch_qpc<T, 48>(p, qpc, grid, threads, smem_bytes, stream);
    case 64: return launch_qpc<T, 64>(p, qpc, grid, threads, smem_bytes, stream);
    case 80: return launch_qpc<T, 80>(p, qpc, grid, threads, smem_bytes, stream);
    case 96: return launch_qpc<T, 96>(p, qpc, grid, threads, smem_bytes, stream);
    case 112: return launch_qpc<T, 112>(p, qpc, grid, threads, smem_bytes, stream);
    case 128: return launch_qpc<T, 128>(p, qpc, grid, threads, smem_bytes, stream);
    case 160: return launch_qpc<T, 160>(p, qpc, grid, threads, smem_bytes, stream);
    case 192: return launch_qpc<T, 192>(p, qpc, grid, threads, smem_bytes, stream);
    case 224: return launch_qpc<T, 224>(p, qpc, grid, threads, smem_bytes, stream);
    case 256: return launch_qpc<T, 256>(p, qpc, grid, threads, smem_bytes, stream);
    case 512: return launch_qpc<T, 512>(p, qpc, grid, threads, smem_bytes, stream);
    default: return fail(VFL_ERR_UNSUPPORTED, "head_dim %d not built", head_dim);
  }
}

}  // namespace vfl
