// Balanced schedule of the tensor-core paged attention kernel (bf16, head_dim 64).
//
// The item grid of paged_attention_tc_kernel (one CTA per request x head group x split) fills
// B200's CTA slots unevenly when a call has few items: 85 requests x 4 head groups are 340 CTAs
// for 444 slots (148 SMs x 3), so 44 SMs carry three items, 104 carry two, and the launch lasts
// as long as the busiest SMs; every CTA also pays its own pipeline start. Here one persistent
// wave of CTAs takes equal runs of the items' 16-token tiles:
//   * the items (request r, head group g) lie end to end in (r, g) order; item (r, g) holds
//     n_r = ceil(L_r / 16) tiles. Of the T tiles in all, CTA c of Ce takes the run
//     [c T / Ce, (c + 1) T / Ce): runs differ by at most one tile;
//   * every CTA reads all lengths and query ranges once into shared memory and derives the same
//     layout with a block-wide prefix sum: no host pass and no extra launch, and a plan captured
//     in a CUDA graph stays valid while the lengths change from step to step;
//   * the producer's ring runs across item boundaries, so the next item's tiles stream in while
//     the consumers finish the current one, and the block-table entries of the next 32 blocks
//     are loaded while the current ones are issued;
//   * a whole item in one run is normalised and stored directly. A piece that a run cut off is
//     stored as an (m, l, acc) partial record of the CTA (slot 0: the piece its run begins
//     with; slot 1: the piece its run ends with); the CTA holding an item's first tile records
//     where the item's pieces went, and a second launch merges them. That launch is a
//     programmatic dependent launch: it starts while this grid drains and waits for it with
//     griddepcontrol.wait.
// Same tile math (tc_consume_tile), fused KV append and bounded waits as the item kernel.
#pragma once

#include "paged_attention_tc.cuh"

namespace vfl {

// Partial record of CTA c's piece `slot`, consumer warp w, query row j: [grid, 2, hpc, kTcRows].
__device__ __forceinline__ int64_t balanced_record(int64_t c, int slot, int w, int j, int hpc) {
  return ((c * 2 + slot) * hpc + w) * kTcRows + j;
}

// The CTA whose run holds global tile t, runs being [c T / ce, (c + 1) T / ce).
__device__ __forceinline__ int balanced_cta_of(int64_t t, int64_t total, int ce) {
  return static_cast<int>(((t + 1) * ce - 1) / total);
}

// One piece of an item: the item's tiles [t_lo, t_hi) that one run holds.
struct BalancedPiece {
  int r, g, n;       // request, head group, the item's tiles
  int t_lo, t_hi;
  int64_t item0;     // the item's first global tile
};

// The pieces of one run, in order, from the shared tile prefix (pref[r + 1] - pref[r] tiles
// per item of request r; G items per request). The producer and every consumer warp walk
// their own copy alike.
struct BalancedWalk {
  const int32_t* pref;
  int G;
  int r;
  int64_t pos, end;

  __device__ __forceinline__ bool next(BalancedPiece& pc) {
    if (pos >= end) return false;
    while ((int64_t)G * pref[r + 1] <= pos) ++r;  // skips requests without tiles
    const int n = pref[r + 1] - pref[r];
    const int64_t req0 = (int64_t)G * pref[r];
    const int g = static_cast<int>((pos - req0) / n);
    const int64_t item0 = req0 + (int64_t)g * n;
    pc.r = r;
    pc.g = g;
    pc.n = n;
    pc.item0 = item0;
    pc.t_lo = static_cast<int>(pos - item0);
    const int64_t stop = item0 + n < end ? item0 + n : end;
    pc.t_hi = static_cast<int>(stop - item0);
    pos = stop;
    return true;
  }
};

// The new positions of a request's query rows in its sequence (fused append): rows [L - nq, L)
// for causal rows, L - 1 for every row otherwise.
__device__ __forceinline__ void balanced_new_range(const AttnParams& p, int L, int nq, int* lo, int* hi) {
  *lo = p.causal ? L - nq : L - 1;
  *hi = L - 1;
}

__device__ __forceinline__ bool balanced_piece_appends(const AttnParams& p, int L, int nq, const BalancedPiece& pc) {
  int lo, hi;
  balanced_new_range(p, L, nq, &lo, &hi);
  return p.new_k != nullptr && hi >= 0 && hi >= pc.t_lo * 16 && lo < pc.t_hi * 16;
}

__global__ void __launch_bounds__(160, 3) paged_attention_tc_balanced_kernel(const AttnParams p,
                                                                              const __grid_constant__ CUtensorMap kmap,
                                                                              const __grid_constant__ CUtensorMap vmap) {
  constexpr int D = 64;
  constexpr int TILE = 16 * D;
  using T = __nv_bfloat16;

  extern __shared__ __align__(1024) uint8_t smem[];
  SmemHeader& hdr = *reinterpret_cast<SmemHeader*>(smem);
  int* s_part = hdr.table;  // block-scan partials [0, 5) and the error flag [7] (no table slice here)
  T* s_kv = reinterpret_cast<T*>(smem + kTcHeaderBytes);
  const int hpc = p.heads_per_cta;
  const int stages = p.stages;
  const int stage_elems = 2 * hpc * TILE;
  const int R = p.num_reqs;
  int32_t* s_pref = reinterpret_cast<int32_t*>(smem + kTcHeaderBytes + (size_t)stages * stage_elems * sizeof(T));
  int32_t* s_lr = s_pref + R + 1;  // clamped length * 16 + query rows (0: no rows, or bad range)
  int32_t* s_qb = s_lr + R;        // first query row

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool producer = warp == hpc;
  const int G = p.num_heads / hpc;
  const int bs = p.block_size;
  const int tpb = bs / 16;

  if (stages < 2 || stages > kMaxStages || R > kBalancedMaxReqs || p.min_tiles < 1) {  // the host checks too
    if (threadIdx.x == 0) report(p.err, VFL_DEVERR_CONTEXT);
    return;
  }
  if (threadIdx.x == 0) s_part[7] = (load_volatile(p.err) & VFL_DEVERR_TIMEOUT) != 0;

  // ---- every request's tiles, length and rows (one coalesced pass)
  const int cap = min(p.table_cols * bs, p.max_seq_len);
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    const int qb = __ldg(p.qsl + r), qe = __ldg(p.qsl + r + 1);
    int L = __ldg(p.seq_lens + r);
    int tiles = 0, lr = 0;
    if (qb < 0 || qe < qb || qe > p.total_q || qe - qb > kTcRows) {
      if (blockIdx.x == 0) report(p.err, VFL_DEVERR_QUERY);
    } else if (qe > qb) {
      if (L > cap) {
        if (blockIdx.x == 0) report(p.err, VFL_DEVERR_CONTEXT);
        L = cap;
      }
      L = max(L, 0);
      tiles = ceil_div(L, 16);
      lr = L * 16 + (qe - qb);
    }
    s_pref[r] = tiles;
    s_lr[r] = lr;
    s_qb[r] = qb;
  }
  __syncthreads();
  if (s_part[7]) return;  // an earlier CTA gave up waiting (one read for the whole CTA)
  // ---- exclusive prefix sum of the tiles: contiguous chunks per thread, then a block scan
  {
    const int per = ceil_div(R, (int)blockDim.x);
    const int lo = min(R, (int)threadIdx.x * per), hi = min(R, lo + per);
    int sum = 0;
    for (int r = lo; r < hi; ++r) sum += s_pref[r];
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    if (lane == 31) s_part[warp] = incl;
    __syncthreads();
    int run = incl - sum;
    for (int w = 0; w < warp; ++w) run += s_part[w];
    for (int r = lo; r < hi; ++r) {
      const int t = s_pref[r];
      s_pref[r] = run;
      run += t;
    }
    if (threadIdx.x == blockDim.x - 1) s_pref[R] = run;
  }
  __syncthreads();

  const int64_t total = (int64_t)G * s_pref[R];
  const int64_t by_min = (total + p.min_tiles - 1) / p.min_tiles;
  const int ce = static_cast<int>(by_min < 1 ? 1 : (by_min < (int64_t)gridDim.x ? by_min : (int64_t)gridDim.x));
  const int c = blockIdx.x;
  if (c >= ce) return;

  // ---- requests without tiles (no rows, a bad range, or length 0): the directory says so, and
  //      rows of length 0 read as zeros, as in the item kernel. Spread over the CTAs by r mod ce.
  for (int r = c; r < R; r += ce) {
    if (s_pref[r + 1] != s_pref[r]) continue;
    for (int g = threadIdx.x; g < G; g += blockDim.x) p.ws_desc[(int64_t)r * G + g] = make_int4(0, 0, 0, 0);
    const int nq = s_lr[r] & 15;
    const int64_t pieces = (int64_t)nq * p.num_heads * (D / 8);
    for (int64_t i = threadIdx.x; i < pieces; i += blockDim.x) {
      const int64_t row = s_qb[r] + i / (p.num_heads * (D / 8));
      const int64_t rest = i - (row - s_qb[r]) * (p.num_heads * (D / 8));
      *reinterpret_cast<uint4*>(static_cast<T*>(p.out) + row * p.out_stride + rest * 8) = make_uint4(0, 0, 0, 0);
    }
  }
  if (total == 0) return;

  const int64_t run_lo = (int64_t)c * total / ce, run_hi = (int64_t)(c + 1) * total / ce;
  int r0 = 0;  // the request holding run_lo: the last r with G * pref[r] <= run_lo
  {
    int lo = 0, hi = R - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((int64_t)G * s_pref[mid] <= run_lo) lo = mid; else hi = mid - 1;
    }
    r0 = lo;
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
    // The tiles of every piece in order. Lane i holds the block-table entry of block b0 + i of
    // the current 32-block chunk; the next chunk's entries load while this one is issued.
    const uint64_t policy = l2_evict_first_policy();
    BalancedWalk walk{s_pref, G, r0, run_lo, run_hi};
    BalancedPiece pc;
    bool have = walk.next(pc);
    int b0 = have ? pc.t_lo / tpb : 0;
    auto load_chunk = [&](const BalancedPiece& q, int base) {
      const int last = (q.t_hi - 1) / tpb;
      int b = 0;
      if (base + lane <= last) {
        b = __ldg(p.table + (int64_t)q.r * p.table_stride + base + lane);
        if (b < 0 || b >= p.num_blocks) {
          report(p.err, VFL_DEVERR_BLOCK_ID);
          b = 0;
        }
      }
      return b;
    };
    int next_phys = have ? load_chunk(pc, b0) : 0;
    // lane 0's unit u sits in stage s of ring round u / stages (counters, no division: the
    // per-tile chain of the issuing thread bounds the tiles in flight)
    int u = 0, s = 0, round = 0, issued = 0, appends_seen = 0;
    const int H = p.num_heads;
    bool stop = false;
    bool piece_start = true;
    bool append_wait = false;  // lane 0: this piece's appended stores not yet waited for
    int first_new_tile = 0;
    while (have && !stop) {
      const int phys_lane = next_phys;
      const int last_blk = (pc.t_hi - 1) / tpb;
      const int chunk_end = min(b0 + 32, last_blk + 1);  // blocks [b0, chunk_end) of this piece
      const bool piece_ends = chunk_end > last_blk;
      // the chunk after this one: the rest of the piece, or the next piece's first blocks
      BalancedPiece nxt = pc;
      BalancedWalk after = walk;
      bool nxt_have = true;
      int nxt_b0 = chunk_end;
      if (piece_ends) {
        nxt_have = after.next(nxt);
        nxt_b0 = nxt_have ? nxt.t_lo / tpb : 0;
      }
      if (nxt_have) next_phys = load_chunk(nxt, nxt_b0);
      if (piece_start) {  // the piece's new K/V (fused append) is stored before its tile loads
        const int lr = s_lr[pc.r];
        const int L = lr >> 4, nq = lr & 15;
        append_wait = balanced_piece_appends(p, L, nq, pc);
        if (append_wait) {
          int lo, hi;
          balanced_new_range(p, L, nq, &lo, &hi);
          first_new_tile = max(lo, pc.t_lo * 16) / 16;  // < t_hi: the piece holds a new position
        }
      }
      const int h0 = pc.g * hpc;
      const int t_from = max(pc.t_lo, b0 * tpb), t_to = min(pc.t_hi, chunk_end * tpb);
      int blk = t_from / tpb, sub_tile = t_from - blk * tpb;  // t == blk * tpb + sub_tile
      for (int t = t_from; t < t_to && !stop; ++t) {
        const int phys = __shfl_sync(0xffffffffu, phys_lane, blk - b0);
        if (lane == 0) {
          if (append_wait && t >= first_new_tile) {
            append_wait = false;
            if (!mbar_wait_bounded(&hdr.appended, appends_seen & 1)) {
              report(p.err, VFL_DEVERR_TIMEOUT);
              hdr.abort = 1;
              stop = true;
            }
            ++appends_seen;
          }
          if (!stop && round > 0 && !mbar_wait_bounded(&hdr.empty[s], (round - 1) & 1)) {
            report(p.err, VFL_DEVERR_TIMEOUT);
            hdr.abort = 1;
            stop = true;
          }
          if (!stop && *reinterpret_cast<volatile int*>(&hdr.abort)) stop = true;
          if (!stop) {  // no proxy fence: consumers only read stages (as in the item kernel)
            T* ks = s_kv + s * stage_elems;
            T* vs = ks + hpc * TILE;
            mbar_arrive_expect_tx(&hdr.full[s], 2u * hpc * TILE * sizeof(T));
            // pool rows [blocks * H * bs, 64]: the tensor maps bound them to int32
            const int row0 = (phys * H + h0) * bs + sub_tile * 16;
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
        }
        stop = __shfl_sync(0xffffffffu, stop, 0);
        if (++sub_tile == tpb) {
          sub_tile = 0;
          ++blk;
        }
      }
      if (piece_ends) {
        pc = nxt;
        walk = after;
        have = nxt_have;
      }
      piece_start = piece_ends;
      b0 = nxt_b0;
    }
    if (lane == 0) griddep_launch_dependents();  // the merge launch may start; it waits for the grid
    __syncwarp();
    __syncthreads();
    if (lane == 0 && *reinterpret_cast<volatile int*>(&hdr.abort)) {
      for (int t = *reinterpret_cast<volatile int*>(&hdr.consumed); t < issued; ++t)
        mbar_wait_bounded(&hdr.full[t % stages], (t / stages) & 1);
    }
    return;
  }

  // ================= consumers: one warp per head of the piece's head group =================
  const TcLane ln(lane);
  const int tq = ln.tq;
  T* p_tile = reinterpret_cast<T*>(smem + kTcPTileOffset) + warp * (kTcRows * 16);
  const uint32_t p_tile_u32 = smem_u32(p_tile);
  BalancedWalk walk{s_pref, G, r0, run_lo, run_hi};
  BalancedPiece pc;
  bool have = walk.next(pc);
  // query fragments of the current piece, loaded one piece ahead
  uint32_t bq_next[4][2];
  if (have) {
    const int nq = s_lr[pc.r] & 15;
    tc_load_query(p, (int64_t)s_qb[pc.r] + ln.g, ln.g < nq, pc.g * hpc + warp, ln, bq_next);
  }
  bool aborted = false;
  int u = 0, s = 0, round = 0;  // unit u sits in stage s of ring round u / stages
  const uint32_t kt0 = smem_u32(s_kv + warp * TILE);
  const uint32_t stage_bytes = stage_elems * sizeof(T);
  const uint32_t v_off = hpc * TILE * sizeof(T);
#pragma unroll 1
  while (have && !aborted) {
    uint32_t bq[4][2];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      bq[kk][0] = bq_next[kk][0];
      bq[kk][1] = bq_next[kk][1];
    }
    BalancedPiece nxt;
    const bool nxt_have = walk.next(nxt);
    if (nxt_have) {
      const int nq_n = s_lr[nxt.r] & 15;
      tc_load_query(p, (int64_t)s_qb[nxt.r] + ln.g, ln.g < nq_n, nxt.g * hpc + warp, ln, bq_next);
    }
    const int h = pc.g * hpc + warp;
    const int lr = s_lr[pc.r];
    const int L = lr >> 4, nq = lr & 15;
    const int q0 = s_qb[pc.r], q_end = q0 + nq;
    if (balanced_piece_appends(p, L, nq, pc)) {
      tc_append_rows(p, q0, nq, q_end, L, h, pc.t_lo * 16, pc.t_hi * 16, warp, lane);
      if (lane == 0) mbar_arrive(&hdr.appended);
    }
    int vis_c[2];
    bool col_on[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = 2 * tq + e;
      col_on[e] = j < nq;
      vis_c[e] = col_on[e] ? max(p.causal ? L - (nq - 1 - j) : L, 0) : 0;
    }
    TcAccum acc;
    acc.reset();
#pragma unroll 1
    for (int t = pc.t_lo; t < pc.t_hi; ++t) {
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
      tc_consume_tile(kt, kt + v_off, bq, col_on, t * 16, vis_c, p.scale_log2, p_tile, p_tile_u32, ln, acc);
      __syncwarp();  // P tile and K/V stage reads done before the next tile reuses them
      if (lane == 0) mbar_arrive(&hdr.empty[s]);
      ++u;
      if (++s == stages) {
        s = 0;
        ++round;
      }
    }
    if (aborted) break;
    acc.reduce_l();
    const bool whole = pc.t_lo == 0 && pc.t_hi == pc.n;
    const int slot = pc.item0 + pc.t_lo == run_lo ? 0 : 1;
    if (whole) {
#pragma unroll
      for (int e = 0; e < 2; ++e)
        if (col_on[e])
          acc.store_output(e, static_cast<T*>(p.out) + (int64_t)(q0 + 2 * tq + e) * p.out_stride + h * D, ln);
    } else {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        if (!col_on[e]) continue;
        const int64_t rec = balanced_record(c, slot, warp, 2 * tq + e, hpc);
        acc.store_partial(e, p.ws_acc + rec * D, p.ws_ml + rec * 2, ln);
      }
    }
    if (pc.t_lo == 0 && warp == 0 && lane == 0) {  // where this item's pieces went
      const int pieces = whole ? 1 : balanced_cta_of(pc.item0 + pc.n - 1, total, ce) - c + 1;
      p.ws_desc[(int64_t)pc.r * G + pc.g] = make_int4(c, slot, pieces, 0);
    }
    pc = nxt;
    have = nxt_have;
  }
  __syncthreads();  // pairs with the producer's barrier (abort bookkeeping)
}

// Merges the pieces of the items the balanced kernel cut: CTA (item, query row j), one warp per
// head of the item's head group. Each piece's (m, l) and the first kPre pieces' partial outputs
// load in one round, then fixed-order sums. Waits for the attention grid with
// griddepcontrol.wait (launched as its programmatic dependent).
__global__ void __launch_bounds__(128) paged_attention_tc_balanced_combine_kernel(const AttnParams p) {
  constexpr int D = 64;
  constexpr int kPre = 8;
  const int hpc = p.heads_per_cta;
  const int G = p.num_heads / hpc;
  const int r = blockIdx.x / G, g = blockIdx.x - r * G, j = blockIdx.y;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = __ldg(p.qsl + r), qe = __ldg(p.qsl + r + 1);  // inputs: read before the wait
  griddep_wait();
  if (w >= hpc || qb < 0 || qe < qb || qe > p.total_q || qe - qb > kTcRows || j >= qe - qb) return;
  // An attention grid that gave up (a timeout in the error word) wrote no directory, or part of
  // one: nothing to merge. No entry may send the reads outside the records of the grid's CTAs.
  if (load_volatile(p.err) & VFL_DEVERR_TIMEOUT) return;
  const int4 d = __ldcg(p.ws_desc + blockIdx.x);
  const int pieces = d.z;
  if (pieces <= 1) return;
  if (d.x < 0 || (d.y != 0 && d.y != 1) || pieces > p.balanced_ctas - d.x) {
    if (threadIdx.x == 0) report(p.err, VFL_DEVERR_CONTEXT);
    return;
  }
  const int h = g * hpc + w;
  // piece i's record: CTA d.x + i, slot d.y for the first piece and 0 after it
  const int64_t first = balanced_record(d.x, d.y, w, j, hpc);
  const int64_t second = balanced_record((int64_t)d.x + 1, 0, w, j, hpc);
  const int64_t stride = balanced_record(1, 0, 0, 0, hpc);  // one CTA further, slot 0
  auto rec = [&](int i) { return i == 0 ? first : second + (i - 1) * stride; };
  const float2* ml = reinterpret_cast<const float2*>(p.ws_ml);
  float2 own = make_float2(-INFINITY, 0.f);  // piece `lane`
  if (lane < pieces) own = __ldcg(ml + rec(lane));
  float pre0[kPre], pre1[kPre];
#pragma unroll
  for (int k = 0; k < kPre; ++k) {
    pre0[k] = pre1[k] = 0.f;
    if (k < pieces) {
      const float* src = p.ws_acc + rec(k) * D;
      pre0[k] = __ldcg(src + lane);
      pre1[k] = __ldcg(src + lane + 32);
    }
  }
  float M = own.x;
  for (int i = lane + 32; i < pieces; i += 32) M = fmaxf(M, __ldcg(ml + rec(i)).x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float o0 = 0.f, o1 = 0.f, lsum = 0.f;
  if (M != -INFINITY) {
    for (int i0 = 0; i0 < pieces; i0 += 32) {
      float wt = 0.f;
      if (i0 + lane < pieces) {
        const float2 v = i0 == 0 ? own : __ldcg(ml + rec(i0 + lane));
        wt = exp2f(v.x - M);
        lsum = fmaf(wt, v.y, lsum);
      }
      const int n = min(32, pieces - i0);
      int k0 = 0;
      if (i0 == 0) {
#pragma unroll
        for (int k = 0; k < kPre; ++k) {
          const float wk = __shfl_sync(0xffffffffu, wt, k);
          if (k < n) {
            o0 = fmaf(wk, pre0[k], o0);
            o1 = fmaf(wk, pre1[k], o1);
          }
        }
        k0 = kPre;
      }
      for (int k = k0; k < n; ++k) {
        const float wk = __shfl_sync(0xffffffffu, wt, k);
        const float* src = p.ws_acc + rec(i0 + k) * D;
        o0 = fmaf(wk, __ldcg(src + lane), o0);
        o1 = fmaf(wk, __ldcg(src + lane + 32), o1);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + (int64_t)(qb + j) * p.out_stride + h * D;
  out[lane] = __float2bfloat16_rn(o0 * inv);
  out[lane + 32] = __float2bfloat16_rn(o1 * inv);
}

}  // namespace vfl
