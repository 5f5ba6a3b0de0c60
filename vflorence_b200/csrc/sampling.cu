// Device-side candidate selection of a decode step (sm_100a).
//
//   row_topk_warp_kernel  (k <= 32) rows x chunks CTAs: one pass over a chunk of a row of a
//                      [rows, vocab] score matrix keeps each warp's best k keys in one list
//                      shared by its lanes (and, for beam search, running maxima and sums of
//                      exponentials); the block's warps merge, and with several chunks per row
//                      row_topk_merge_kernel merges the chunks. The top-k become log-probs
//                      shifted by the row's cumulative log-prob. Replaces logits.float(),
//                      log_softmax, topk and the cum add of the reference's _sample /
//                      _beam_search (vflorence/engine/model_runner.py:370-399) and the greedy
//                      argmax (:379).
//   row_topk_kernel    (33 <= k <= 64) one CTA per row, per-thread register lists.
//   beam_merge_kernel  one warp per request: the request's rows' candidates ordered as a
//                      stable descending sort of the rows' lists in row order
//                      (model_runner.py:401-410), the best `keep` written out.
//
// Keys are 64-bit: the order-preserving image of the float value in the high word and the
// complement of the index (or list position) in the low word, so every key is distinct and a
// larger key is a larger value, or an equal value at a lower index - the tie rule of argmax.
#include <cfloat>
#include <cmath>

#include "common.cuh"

namespace vfl {
namespace {

constexpr int kTopkThreads = 256;
constexpr int kMaxK = 64;

__device__ __forceinline__ uint32_t ordered_bits(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float from_ordered_bits(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

__device__ __forceinline__ uint64_t make_key(float v, uint32_t idx) {
  return (static_cast<uint64_t>(ordered_bits(v)) << 32) | static_cast<uint32_t>(~idx);
}

__device__ __forceinline__ float key_value(uint64_t key) { return from_ordered_bits(static_cast<uint32_t>(key >> 32)); }
__device__ __forceinline__ uint32_t key_index(uint64_t key) { return ~static_cast<uint32_t>(key); }

__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int mask) {
  return __shfl_xor_sync(0xffffffffu, v, mask);
}

// Inserts `key` into a descending register list (one bubble pass; the smallest drops out).
template <int K>
__device__ __forceinline__ void list_insert(uint64_t (&list)[K], uint64_t key) {
#pragma unroll
  for (int q = 0; q < K; ++q) {
    const uint64_t hi = list[q] > key ? list[q] : key;
    key = list[q] > key ? key : list[q];
    list[q] = hi;
  }
}

// Pops the head of a descending register list.
template <int K>
__device__ __forceinline__ void list_pop(uint64_t (&list)[K]) {
#pragma unroll
  for (int q = 0; q + 1 < K; ++q) list[q] = list[q + 1];
  list[K - 1] = 0;
}

// The warp's best K keys over its lanes' sorted lists, written by lane 0 to `dst[0..K)`.
template <int K>
__device__ __forceinline__ void warp_merge(uint64_t (&list)[K], uint64_t* dst, int lane) {
#pragma unroll 1
  for (int j = 0; j < K; ++j) {
    uint64_t best = list[0];
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const uint64_t o = shfl_xor_u64(best, m);
      best = o > best ? o : best;
    }
    if (lane == 0) dst[j] = best;
    if (best != 0 && list[0] == best) list_pop(list);
  }
}

template <typename T>
struct Vec16;
template <>
struct Vec16<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void load(const float* p, float (&v)[N]) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  }
};
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void load(const __nv_bfloat16* p, float (&v)[N]) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};

__device__ __forceinline__ float to_float(float x) { return x; }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

struct RowStats {
  float m;  // running max
  float s;  // sum of exp(x - m)
};

__device__ __forceinline__ void stats_add(RowStats& st, float x) {
  if (x > st.m) {
    st.s = st.s * expf(st.m - x) + 1.0f;
    st.m = x;
  } else if (x != -INFINITY) {
    st.s += expf(x - st.m);
  }
}

__device__ __forceinline__ RowStats stats_merge(RowStats a, RowStats b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.0f};
  return {m, a.s * expf(a.m - m) + b.s * expf(b.m - m)};
}

template <typename T, int K, bool kLogSoftmax>
__device__ __forceinline__ void visit(uint64_t (&list)[K], RowStats& st, float x, uint32_t idx) {
  if (kLogSoftmax) stats_add(st, x);
  const uint64_t key = make_key(x, idx);
  if (key > list[K - 1]) list_insert(list, key);
}

template <typename T, int K, bool kLogSoftmax>
__global__ void __launch_bounds__(kTopkThreads) row_topk_kernel(const T* __restrict__ scores, int64_t vocab,
                                                                 int64_t row_stride, const float* __restrict__ offset,
                                                                 int k, float* __restrict__ values,
                                                                 int32_t* __restrict__ indices) {
  __shared__ uint64_t warp_best[kTopkThreads / 32][K];
  __shared__ uint64_t row_best[K];
  __shared__ RowStats warp_stats[kTopkThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t r = blockIdx.x;
  const T* x = scores + r * row_stride;

  uint64_t list[K];
#pragma unroll
  for (int q = 0; q < K; ++q) list[q] = 0;
  RowStats st{-INFINITY, 0.0f};

  // head elements up to a 16-byte boundary, then 16-byte vectors, then the tail
  using V = Vec16<T>;
  const int64_t mis = (reinterpret_cast<uintptr_t>(x) & 15u) / sizeof(T);
  int64_t head = mis == 0 ? 0 : (16 / (int64_t)sizeof(T)) - mis;
  head = head < vocab ? head : vocab;
  for (int64_t i = tid; i < head; i += kTopkThreads) visit<T, K, kLogSoftmax>(list, st, to_float(x[i]), (uint32_t)i);
  const int64_t nvec = (vocab - head) / V::N;
  const T* xv = x + head;
  // U independent 16-byte loads in flight per thread before any of them is consumed (one CTA
  // per row leaves few warps per SM, so the row streams only if each thread keeps several
  // loads outstanding); fewer for the wide-K lists, whose registers are already committed
  constexpr int U = K <= 16 ? 32 / V::N : (K <= 32 ? (V::N >= 8 ? 1 : 8 / V::N) : 1);
  for (int64_t v0 = tid; v0 < nvec; v0 += (int64_t)kTopkThreads * U) {
    float e[U][V::N];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + (int64_t)u * kTopkThreads;
      if (v < nvec) V::load(xv + v * V::N, e[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + (int64_t)u * kTopkThreads;
      if (v < nvec) {
#pragma unroll
        for (int q = 0; q < V::N; ++q)
          visit<T, K, kLogSoftmax>(list, st, e[u][q], (uint32_t)(head + v * V::N + q));
      }
    }
  }
  for (int64_t i = head + nvec * V::N + tid; i < vocab; i += kTopkThreads)
    visit<T, K, kLogSoftmax>(list, st, to_float(x[i]), (uint32_t)i);

  // warp, then block: the row's top K keys (and the row's max / sum of exponentials)
  warp_merge(list, warp_best[warp], lane);
  if (kLogSoftmax) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      RowStats o{__shfl_xor_sync(0xffffffffu, st.m, m), __shfl_xor_sync(0xffffffffu, st.s, m)};
      st = stats_merge(st, o);
    }
  }
  if (lane == 0) warp_stats[warp] = st;
  __syncthreads();
  if (warp != 0) return;
  constexpr int kWarps = kTopkThreads / 32;
#pragma unroll
  for (int q = 0; q < K; ++q) list[q] = lane < kWarps ? warp_best[lane][q] : 0;
  __syncwarp();
  warp_merge(list, row_best, lane);
  __syncwarp();
  float shift = 0.0f, lse = 0.0f;
  if (kLogSoftmax) {
    RowStats all = warp_stats[0];
    for (int w = 1; w < kWarps; ++w) all = stats_merge(all, warp_stats[w]);
    shift = all.m;
    lse = logf(all.s);
  }
  const float add = offset != nullptr ? offset[r] : 0.0f;
  if (lane == 0) {
    for (int j = 0; j < k; ++j) {
      float v = key_value(row_best[j]);
      if (kLogSoftmax) v = (v - shift) - lse;  // log_softmax as (x - max) - log(sum)
      values[r * k + j] = v + add;
      indices[r * k + j] = (int32_t)key_index(row_best[j]);
    }
  }
}

// k <= 32: each warp keeps ONE shared list, lane j holding the warp's j-th best key, so an
// element costs a float compare with the warp's k-th value and a ballot; the rare winners are
// inserted one at a time by the whole warp. Every lane walks its range in the same order
// (warp-uniform loops, out-of-range lanes offer nothing). For beam search each lane also keeps
// a running max and sum of exp(x - max), updated once per batch of its elements.
struct WarpList {
  uint64_t mine = 0;  // lane j < k: the warp's j-th best key (0 = empty)
  uint64_t thr = 0;   // the warp's k-th best key (0 while the list is not full)
  float thr_val = 0.0f;

  __device__ __forceinline__ static uint64_t shfl_u64(uint64_t v, int src) {
    return __shfl_sync(0xffffffffu, v, src);
  }

  // `pass`: this lane's element may beat the k-th key (a cheap superset test); `key` is only
  // read for such lanes
  __device__ __forceinline__ void offer_if(bool pass, uint64_t key, int lane, int k) {
    unsigned ball = __ballot_sync(0xffffffffu, pass && key > thr);
    while (ball) {
      const int src = __ffs(ball) - 1;
      ball &= ball - 1;
      const uint64_t cand = shfl_u64(key, src);
      if (cand > thr) {  // uniform: cand and thr are the same in every lane
        const int pos = __popc(__ballot_sync(0xffffffffu, lane < k && mine > cand));
        const uint64_t up = __shfl_up_sync(0xffffffffu, mine, 1);
        if (lane < k) mine = lane > pos ? up : (lane == pos ? cand : mine);
        thr = shfl_u64(mine, k - 1);
        thr_val = key_value(thr);
      }
    }
  }

  __device__ __forceinline__ bool may_win(float x) const { return thr == 0 || !(x < thr_val); }

  __device__ __forceinline__ void offer_value(bool ok, float x, uint32_t idx, int lane, int k) {
    const bool pass = ok && may_win(x);
    offer_if(pass, pass ? make_key(x, idx) : 0ull, lane, k);
  }
};

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxChunks = 16;
constexpr int64_t kMinChunkElems = 4096;

// What one CTA of a split row leaves for the merge: its best keys and its (max, sum of exp).
struct TopkPartial {
  uint64_t keys[32];
  float m, s;
};

// Chunks per row: as many as one wave of CTAs holds (3 per SM), chunks of at least
// kMinChunkElems elements; a second partial wave costs more than the extra parallelism gives.
int topk_chunks(int64_t rows, int64_t vocab, int k) {
  if (k > 32 || rows <= 0) return 1;
  int64_t c = (int64_t)kNumSMs * 3 / rows;
  const int64_t by_len = vocab / kMinChunkElems;
  c = c < by_len ? c : by_len;
  return (int)(c < 1 ? 1 : (c > kMaxChunks ? kMaxChunks : c));
}

// adds a lane's batch (its valid values, batch maximum `bm`) to its (max, sum of exp) with one
// rescale per batch
__device__ __forceinline__ void stats_rescale(RowStats& st, float bm) {
  if (bm > st.m) {
    st.s *= exp2_approx((st.m - bm) * kLog2e);
    st.m = bm;
  }
}

__device__ __forceinline__ void write_row(float* values, int32_t* indices, const float* offset, int64_t r, int k,
                                          int lane, uint64_t key, bool log_softmax, float shift, float lse) {
  if (lane < k) {
    float v = key_value(key);
    if (log_softmax) v = (v - shift) - lse;  // log_softmax as (x - max) - log(sum)
    values[r * k + lane] = v + (offset != nullptr ? offset[r] : 0.0f);
    indices[r * k + lane] = (int32_t)key_index(key);
  }
}

// The chunk a CTA walks: a contiguous range of the row's 16-byte vectors; chunk 0 also takes the
// ragged head, the last chunk the ragged tail (fewer than 8 elements each, warp 0).
template <typename T>
struct ChunkWalk {
  using V = Vec16<T>;
  static constexpr int U = 32 / V::N;  // a lane's batch: 32 elements, U 16-byte loads in flight
  const T* x;
  const T* xv;
  int64_t vocab, head, tail0, vbegin, vend;
  bool first, last;

  __device__ ChunkWalk(const T* row, int64_t vocab_, int chunk, int chunks) : x(row), vocab(vocab_) {
    const int64_t mis = (reinterpret_cast<uintptr_t>(row) & 15u) / sizeof(T);
    head = mis == 0 ? 0 : (16 / (int64_t)sizeof(T)) - mis;
    head = head < vocab ? head : vocab;
    const int64_t nvec = (vocab - head) / V::N;
    tail0 = head + nvec * V::N;
    xv = x + head;
    const int64_t per = ceil_div(nvec, (int64_t)chunks);
    vbegin = chunk * per;
    vend = vbegin + per < nvec ? vbegin + per : nvec;
    first = chunk == 0;
    last = chunk == chunks - 1;
  }

  // f(ok, values[U][N], first element index of each of the U vectors) once per batch, the same
  // number of times in every lane of a warp; then the ragged ends for warp 0 (one value a lane)
  template <typename F, typename G>
  __device__ __forceinline__ void walk(int warp, int lane, F&& batch, G&& single) const {
    for (int64_t base = vbegin + (int64_t)warp * 32; base < vend; base += (int64_t)kTopkThreads * U) {
      float e[U][V::N];
      bool ok[U];
      int64_t idx[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t v = base + lane + (int64_t)u * kTopkThreads;
        ok[u] = v < vend;
        idx[u] = head + v * V::N;
        if (ok[u]) V::load(xv + v * V::N, e[u]);
      }
      batch(ok, e, idx);
    }
    if (warp == 0) {
      for (int part = 0; part < 2; ++part) {
        if ((part == 0 && !first) || (part == 1 && !last)) continue;
        const int64_t begin = part == 0 ? 0 : tail0, end = part == 0 ? head : vocab;
        const bool ok1 = begin + lane < end;
        single(ok1, ok1 ? to_float(x[begin + lane]) : -INFINITY, begin + lane);
      }
    }
  }
};

// grid: rows x chunks, two passes over the CTA's chunk.
//  pass 1: each lane folds its batches into (max, sum of exp) and offers only the batch maximum
//          to its warp's list; the k-th largest batch maximum of the CTA, T, is a lower bound of
//          the chunk's k-th largest value (batch maxima are distinct elements of the chunk).
//  pass 2: the chunk again (now from L2): one compare per element, one ballot per batch; only
//          batches holding a value >= T insert into the candidate lists.
// With one chunk the CTA writes the row's result, otherwise its TopkPartial.
template <typename T, bool kLogSoftmax>
__global__ void __launch_bounds__(kTopkThreads, 3) row_topk_warp_kernel(const T* __restrict__ scores, int64_t vocab,
                                                                     int64_t row_stride,
                                                                     const float* __restrict__ offset, int k,
                                                                     int chunks, float* __restrict__ values,
                                                                     int32_t* __restrict__ indices,
                                                                     TopkPartial* __restrict__ partials) {
  constexpr int kWarps = kTopkThreads / 32;
  using W = ChunkWalk<T>;
  __shared__ uint64_t warp_best[kWarps][32];
  __shared__ RowStats warp_stats[kWarps];
  __shared__ float s_threshold;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t r = blockIdx.x / chunks;
  const int chunk = blockIdx.x - (int)(r * chunks);
  const W walk(scores + r * row_stride, vocab, chunk, chunks);

  // ---- pass 1: statistics and batch maxima
  WarpList maxima;
  RowStats st{-INFINITY, 0.0f};
  walk.walk(
      warp, lane,
      [&](const bool (&ok)[W::U], const float (&e)[W::U][W::V::N], const int64_t (&idx)[W::U]) {
        float bm = -INFINITY;
        bool any = false;
#pragma unroll
        for (int u = 0; u < W::U; ++u)
          if (ok[u]) {
            any = true;
#pragma unroll
            for (int q = 0; q < W::V::N; ++q) bm = fmaxf(bm, e[u][q]);
          }
        if (kLogSoftmax && any) {
          stats_rescale(st, bm);
          if (st.m != -INFINITY) {
            float add = 0.0f;
#pragma unroll
            for (int u = 0; u < W::U; ++u)
              if (ok[u]) {
#pragma unroll
                for (int q = 0; q < W::V::N; ++q) add += exp2_approx((e[u][q] - st.m) * kLog2e);
              }
            st.s += add;
          }
        }
        maxima.offer_value(any, bm, (uint32_t)idx[0], lane, k);
      },
      [&](bool ok1, float v, int64_t i) {
        if (kLogSoftmax && ok1) {
          stats_rescale(st, v);
          if (st.m != -INFINITY) st.s += exp2_approx((v - st.m) * kLog2e);
        }
        maxima.offer_value(ok1, v, (uint32_t)i, lane, k);
      });
  if (lane < k) warp_best[warp][lane] = maxima.mine;
  if (kLogSoftmax) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      RowStats o{__shfl_xor_sync(0xffffffffu, st.m, m), __shfl_xor_sync(0xffffffffu, st.s, m)};
      st = stats_merge(st, o);
    }
    if (lane == 0) warp_stats[warp] = st;
  }
  __syncthreads();
  if (warp == 0) {
    for (int w = 1; w < kWarps; ++w) {
      const uint64_t key = lane < k ? warp_best[w][lane] : 0ull;
      maxima.offer_if(key != 0, key, lane, k);
    }
    if (lane == 0) s_threshold = maxima.thr == 0 ? -INFINITY : key_value(maxima.thr);
  }
  __syncthreads();
  const float thr = s_threshold;

  // ---- pass 2: every value >= T competes
  WarpList cand;
  walk.walk(
      warp, lane,
      [&](const bool (&ok)[W::U], const float (&e)[W::U][W::V::N], const int64_t (&idx)[W::U]) {
        bool any = false;
#pragma unroll
        for (int u = 0; u < W::U; ++u)
#pragma unroll
          for (int q = 0; q < W::V::N; ++q) any |= ok[u] && e[u][q] >= thr;
        if (__ballot_sync(0xffffffffu, any) == 0u) return;
#pragma unroll
        for (int u = 0; u < W::U; ++u)
#pragma unroll
          for (int q = 0; q < W::V::N; ++q)
            cand.offer_value(ok[u] && e[u][q] >= thr, e[u][q], (uint32_t)(idx[u] + q), lane, k);
      },
      [&](bool ok1, float v, int64_t i) { cand.offer_value(ok1 && v >= thr, v, (uint32_t)i, lane, k); });

  __syncthreads();  // warp_best is reused
  if (lane < k) warp_best[warp][lane] = cand.mine;
  __syncthreads();
  if (warp != 0) return;
  for (int w = 1; w < kWarps; ++w) {
    const uint64_t key = lane < k ? warp_best[w][lane] : 0ull;
    cand.offer_if(key != 0, key, lane, k);
  }
  RowStats all{-INFINITY, 0.0f};
  if (kLogSoftmax) {
    all = warp_stats[0];
    for (int w = 1; w < kWarps; ++w) all = stats_merge(all, warp_stats[w]);
  }
  if (chunks == 1) {
    write_row(values, indices, offset, r, k, lane, cand.mine, kLogSoftmax, all.m, kLogSoftmax ? logf(all.s) : 0.0f);
  } else {
    TopkPartial& part = partials[r * chunks + chunk];
    part.keys[lane] = lane < k ? cand.mine : 0ull;
    if (lane == 0) {
      part.m = all.m;
      part.s = all.s;
    }
  }
}

// One warp per row: the row's chunk partials merged into its final top-k.
template <bool kLogSoftmax>
__global__ void row_topk_merge_kernel(const TopkPartial* __restrict__ partials, int chunks, const float* offset,
                                      int k, float* __restrict__ values, int32_t* __restrict__ indices) {
  const int lane = threadIdx.x;
  const int64_t r = blockIdx.x;
  WarpList wl;
  RowStats all{-INFINITY, 0.0f};
  for (int c = 0; c < chunks; ++c) {
    const TopkPartial& part = partials[r * chunks + c];
    const uint64_t key = lane < k ? part.keys[lane] : 0ull;
    wl.offer_if(key != 0, key, lane, k);
    if (kLogSoftmax) all = stats_merge(all, RowStats{part.m, part.s});
  }
  write_row(values, indices, offset, r, k, lane, wl.mine, kLogSoftmax, all.m, kLogSoftmax ? logf(all.s) : 0.0f);
}

// One warp per request group: its rows (found by group id, placed by rank), then `keep` rounds
// of a warp arg-max over the rows' candidate lists.
__global__ void beam_merge_kernel(const float* __restrict__ values, const int32_t* __restrict__ indices,
                                  int64_t rows, int k, const int32_t* __restrict__ groups,
                                  const int32_t* __restrict__ ranks, int num_groups, int keep,
                                  int32_t* __restrict__ out) {
  constexpr int kMaxRows = 64;
  __shared__ int32_t row_of[4][kMaxRows];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int g = blockIdx.x * 4 + wib;
  if (g >= num_groups) return;
  int32_t* my = row_of[wib];
  for (int i = lane; i < kMaxRows; i += 32) my[i] = -1;
  __syncwarp();
  int count = 0;
  for (int64_t base = 0; base < rows; base += 32) {
    const int64_t i = base + lane;
    const bool mine = i < rows && groups[i] == g;
    if (mine) {
      const int rk = ranks[i];
      if (rk >= 0 && rk < kMaxRows) my[rk] = (int32_t)i;
    }
    count += __popc(__ballot_sync(0xffffffffu, mine));
  }
  __syncwarp();
  if (count > kMaxRows) count = kMaxRows;
  const int total = count * k;
  uint64_t prev = ~0ull;
  int32_t* out_row = out;
  int32_t* out_tok = out + (int64_t)num_groups * keep;
  int32_t* out_val = out + 2 * (int64_t)num_groups * keep;
  for (int j = 0; j < keep; ++j) {
    uint64_t best = 0;
    for (int c = lane; c < total; c += 32) {
      const int rk = c / k, q = c % k;
      const int32_t row = my[rk];
      if (row < 0) continue;
      const uint64_t key = make_key(values[(int64_t)row * k + q], (uint32_t)c);
      if (key < prev && key > best) best = key;
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const uint64_t o = shfl_xor_u64(best, m);
      best = o > best ? o : best;
    }
    if (lane == 0) {
      const int64_t o = (int64_t)g * keep + j;
      if (best == 0) {
        out_row[o] = -1;
        out_tok[o] = 0;
        out_val[o] = (int32_t)__float_as_uint(-INFINITY);
      } else {
        const int c = (int)key_index(best);
        const int32_t row = my[c / k];
        out_row[o] = row;
        out_tok[o] = indices[(int64_t)row * k + c % k];
        out_val[o] = (int32_t)__float_as_uint(values[(int64_t)row * k + c % k]);
      }
    }
    prev = best;
  }
}

template <typename T, int K>
int launch_topk_k(const T* scores, int64_t rows, int64_t vocab, int64_t stride, int log_softmax, const float* offset,
                  int k, float* values, int32_t* indices, cudaStream_t s) {
  if (log_softmax)
    row_topk_kernel<T, K, true><<<(unsigned)rows, kTopkThreads, 0, s>>>(scores, vocab, stride, offset, k, values,
                                                                        indices);
  else
    row_topk_kernel<T, K, false><<<(unsigned)rows, kTopkThreads, 0, s>>>(scores, vocab, stride, offset, k, values,
                                                                         indices);
  return cuda_status(cudaGetLastError(), "row_topk launch");
}

template <typename T>
int launch_topk(const T* scores, int64_t rows, int64_t vocab, int64_t stride, int log_softmax, const float* offset,
                int k, float* values, int32_t* indices, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  if (k > 32) return launch_topk_k<T, 64>(scores, rows, vocab, stride, log_softmax, offset, k, values, indices, s);
  const int chunks = topk_chunks(rows, vocab, k);
  TopkPartial* partials = nullptr;
  if (chunks > 1) {
    const size_t need = (size_t)rows * chunks * sizeof(TopkPartial);
    if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0)
      return fail(VFL_ERR_WORKSPACE, "row_topk: needs %zu workspace bytes (16-byte aligned), got %zu", need,
                  workspace_bytes);
    partials = static_cast<TopkPartial*>(workspace);
  }
  const unsigned grid = (unsigned)(rows * chunks);
  if (log_softmax)
    row_topk_warp_kernel<T, true><<<grid, kTopkThreads, 0, s>>>(scores, vocab, stride, offset, k, chunks, values,
                                                                indices, partials);
  else
    row_topk_warp_kernel<T, false><<<grid, kTopkThreads, 0, s>>>(scores, vocab, stride, offset, k, chunks, values,
                                                                 indices, partials);
  int st = cuda_status(cudaGetLastError(), "row_topk launch");
  if (st || chunks == 1) return st;
  if (log_softmax)
    row_topk_merge_kernel<true><<<(unsigned)rows, 32, 0, s>>>(partials, chunks, offset, k, values, indices);
  else
    row_topk_merge_kernel<false><<<(unsigned)rows, 32, 0, s>>>(partials, chunks, offset, k, values, indices);
  return cuda_status(cudaGetLastError(), "row_topk merge launch");
}

}  // namespace
}  // namespace vfl

using namespace vfl;

extern "C" size_t vfl_row_topk_workspace_size(int64_t rows, int64_t vocab, int32_t k) {
  const int chunks = topk_chunks(rows, vocab, k);
  return chunks > 1 ? (size_t)rows * chunks * sizeof(TopkPartial) : 0;
}

extern "C" int vfl_row_topk(const void* scores, int32_t dtype, int64_t rows, int64_t vocab, int64_t row_stride,
                            int32_t log_softmax, const float* row_offset, int32_t k, float* values,
                            int32_t* indices, void* workspace, size_t workspace_bytes, void* stream) {
  if (!dtype_ok(dtype)) return fail(VFL_ERR_UNSUPPORTED, "row_topk: dtype %d is not float32 or bfloat16", dtype);
  if (rows < 0 || rows > INT32_MAX / kMaxChunks || vocab < 1 || vocab > INT32_MAX || row_stride < vocab)
    return fail(VFL_ERR_INVALID_ARGUMENT, "row_topk: rows %lld, vocab %lld, row stride %lld", (long long)rows,
                (long long)vocab, (long long)row_stride);
  if (k < 1 || k > kMaxK || k > vocab)
    return fail(VFL_ERR_UNSUPPORTED, "row_topk: k = %d outside [1, min(%d, vocab)]", k, kMaxK);
  if (rows == 0) return VFL_OK;
  if (scores == nullptr || values == nullptr || indices == nullptr)
    return fail(VFL_ERR_INVALID_ARGUMENT, "row_topk: NULL pointer");
  const size_t es = dtype_size(dtype);
  if ((reinterpret_cast<uintptr_t>(scores) % es) != 0)
    return fail(VFL_ERR_INVALID_ARGUMENT, "row_topk: scores not aligned to their element size");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == VFL_DTYPE_F32)
    return launch_topk(static_cast<const float*>(scores), rows, vocab, row_stride, log_softmax, row_offset, k,
                       values, indices, workspace, workspace_bytes, s);
  return launch_topk(static_cast<const __nv_bfloat16*>(scores), rows, vocab, row_stride, log_softmax, row_offset, k,
                     values, indices, workspace, workspace_bytes, s);
}

extern "C" int vfl_beam_merge(const float* values, const int32_t* indices, int64_t rows, int32_t k,
                              const int32_t* groups, const int32_t* ranks, int32_t num_groups, int32_t keep,
                              int32_t* out, void* stream) {
  if (rows < 0 || rows > INT32_MAX || k < 1 || k > kMaxK || num_groups < 0 || keep < 1 ||
      (int64_t)keep * num_groups > INT32_MAX)
    return fail(VFL_ERR_INVALID_ARGUMENT, "beam_merge: rows %lld, k %d, groups %d, keep %d", (long long)rows, k,
                num_groups, keep);
  if ((int64_t)64 * k >= (1ll << 31)) return fail(VFL_ERR_INVALID_ARGUMENT, "beam_merge: k too large");
  if (num_groups == 0) return VFL_OK;
  if (values == nullptr || indices == nullptr || groups == nullptr || ranks == nullptr || out == nullptr)
    return fail(VFL_ERR_INVALID_ARGUMENT, "beam_merge: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  beam_merge_kernel<<<(unsigned)((num_groups + 3) / 4), 128, 0, s>>>(values, indices, rows, k, groups, ranks,
                                                                      num_groups, keep, out);
  return cuda_status(cudaGetLastError(), "beam_merge launch");
}

namespace vfl {
namespace {

// One CTA per born child: tokens[child, :] = tokens[parent, :] with tokens[child, pos] = token.
// The runtime hands children slots off its free stack while every parent still holds its own,
// so no child row is a parent row of the same step and one pass is enough.
__global__ void __launch_bounds__(128) fork_token_rows_kernel(int32_t* tokens, int64_t row_stride, int32_t num_rows,
                                                              int32_t width, const int32_t* born, int32_t num_born,
                                                              unsigned int* err) {
  const int i = blockIdx.x;
  const int32_t parent = __ldg(born + i), child = __ldg(born + num_born + i);
  const int32_t pos = __ldg(born + 2 * (int64_t)num_born + i), token = __ldg(born + 3 * (int64_t)num_born + i);
  if (parent < 0 || parent >= num_rows || child < 0 || child >= num_rows || parent == child || pos < 0 ||
      pos >= width) {
    if (threadIdx.x == 0) report(err, VFL_DEVERR_SLOT);
    return;
  }
  const int32_t* src = tokens + parent * row_stride;
  int32_t* dst = tokens + child * row_stride;
  for (int c = threadIdx.x; c < width; c += blockDim.x) dst[c] = c == pos ? token : src[c];
}

}  // namespace
}  // namespace vfl

extern "C" int vfl_fork_token_rows(int32_t* tokens, int64_t row_stride, int32_t num_rows, int32_t width,
                                   const int32_t* born, int32_t num_born, void* stream) {
  if (num_rows < 0 || width < 1 || row_stride < width || num_born < 0 || num_born > (1 << 30))
    return fail(VFL_ERR_INVALID_ARGUMENT, "fork_token_rows: rows %d, width %d, row_stride %lld, born %d", num_rows,
                width, (long long)row_stride, num_born);
  if (num_born == 0) return VFL_OK;
  if (tokens == nullptr || born == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "fork_token_rows: NULL pointer");
  unsigned int* err = nullptr;
  int st = device_error_word(&err);
  if (st) return st;
  fork_token_rows_kernel<<<(unsigned)num_born, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      tokens, row_stride, num_rows, width, born, num_born, err);
  return cuda_status(cudaGetLastError(), "fork_token_rows launch");
}
