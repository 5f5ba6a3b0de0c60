// Device-side candidate selection of a decode step (sm_100a).
//
//   row_topk_kernel    one CTA per row of a [rows, vocab] score matrix: a single pass over the
//                      row keeps every thread's best K keys in registers (and, for beam search,
//                      the row's running max and sum of exponentials), then warp and block
//                      merges give the row's top-k, turned into log-probs and shifted by the
//                      row's cumulative log-prob. Replaces logits.float(), log_softmax, topk and
//                      the cum add of the reference's _sample / _beam_search
//                      (vflorence/engine/model_runner.py:370-399) and the greedy argmax (:379).
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
  for (int64_t v = tid; v < nvec; v += kTopkThreads) {
    float e[V::N];
    V::load(xv + v * V::N, e);
#pragma unroll
    for (int q = 0; q < V::N; ++q)
      visit<T, K, kLogSoftmax>(list, st, e[q], (uint32_t)(head + v * V::N + q));
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
                int k, float* values, int32_t* indices, cudaStream_t s) {
  if (k <= 1) return launch_topk_k<T, 1>(scores, rows, vocab, stride, log_softmax, offset, k, values, indices, s);
  if (k <= 2) return launch_topk_k<T, 2>(scores, rows, vocab, stride, log_softmax, offset, k, values, indices, s);
  if (k <= 4) return launch_topk_k<T, 4>(scores, rows, vocab, stride, log_softmax, offset, k, values, indices, s);
  if (k <= 8) return launch_topk_k<T, 8>(scores, rows, vocab, stride, log_softmax, offset, k, values, indices, s);
  if (k <= 16) return launch_topk_k<T, 16>(scores, rows, vocab, stride, log_softmax, offset, k, values, indices, s);
  if (k <= 32) return launch_topk_k<T, 32>(scores, rows, vocab, stride, log_softmax, offset, k, values, indices, s);
  return launch_topk_k<T, 64>(scores, rows, vocab, stride, log_softmax, offset, k, values, indices, s);
}

}  // namespace
}  // namespace vfl

using namespace vfl;

extern "C" int vfl_row_topk(const void* scores, int32_t dtype, int64_t rows, int64_t vocab, int64_t row_stride,
                            int32_t log_softmax, const float* row_offset, int32_t k, float* values,
                            int32_t* indices, void* stream) {
  if (!dtype_ok(dtype)) return fail(VFL_ERR_UNSUPPORTED, "row_topk: dtype %d is not float32 or bfloat16", dtype);
  if (rows < 0 || rows > INT32_MAX || vocab < 1 || vocab > INT32_MAX || row_stride < vocab)
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
                       values, indices, s);
  return launch_topk(static_cast<const __nv_bfloat16*>(scores), rows, vocab, row_stride, log_softmax, row_offset, k,
                     values, indices, s);
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
