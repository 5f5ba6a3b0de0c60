// KV-cache maintenance kernels of the paged path:
//   vfl_reshape_and_cache  - KV append by slot mapping (vflorence/layers/attention.py:55-57,
//                            vflorence/engine/model_runner.py:252-259)
//   vfl_copy_blocks        - copy-on-write block copies, all layers, one launch
//                            (vflorence/engine/model_runner.py:162-167)
//   vfl_prepare_decode     - per-step slot mapping / context lengths on the device
//                            (vflorence/engine/model_runner.py:290-306)
//   vfl_paged_slots        - encoder slots from a request's pages (model_runner.py:240-242)
// All are HBM-bound byte movers: 16-byte vector accesses, grids sized to the 148 SMs.
#include "common.cuh"

namespace vfl {
namespace {

// One thread per 16-byte vector of a (token, head) row; rows are `row_vecs` vectors long.
__global__ void __launch_bounds__(256) reshape_and_cache_kernel(
    const uint8_t* __restrict__ key, const uint8_t* __restrict__ value, uint4* __restrict__ k_cache,
    uint4* __restrict__ v_cache, const int64_t* __restrict__ slots, int64_t num_tokens,
    int num_heads, int row_vecs, int block_size, int64_t num_blocks, int64_t key_stride_bytes,
    int64_t value_stride_bytes, unsigned int* err) {
  const int64_t total = num_tokens * num_heads * row_vecs;
  const int64_t capacity = num_blocks * block_size;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c = static_cast<int>(i % row_vecs);
    const int64_t th = i / row_vecs;
    const int h = static_cast<int>(th % num_heads);
    const int64_t t = th / num_heads;
    const int64_t slot = __ldg(slots + t);
    if (slot < 0) continue;  // padding token: nothing to store
    if (slot >= capacity) {
      if (h == 0 && c == 0) report(err, VFL_DEVERR_SLOT);
      continue;
    }
    const int64_t blk = slot / block_size;
    const int64_t off = slot - blk * block_size;
    const int64_t src_off = (int64_t)(h * row_vecs + c) * 16;
    const uint4 kv = ldg_nc_v4(key + t * key_stride_bytes + src_off);
    const uint4 vv = ldg_nc_v4(value + t * value_stride_bytes + src_off);
    const int64_t dst = ((blk * num_heads + h) * block_size + off) * row_vecs + c;
    k_cache[dst] = kv;
    v_cache[dst] = vv;
  }
}

struct CopyLayers {
  uint4* k[VFL_MAX_COPY_LAYERS];
  uint4* v[VFL_MAX_COPY_LAYERS];
};

// blockIdx.x = pair, blockIdx.y = layer * 2 + (0: K, 1: V). Each CTA moves one whole block.
constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 4;
__global__ void __launch_bounds__(kCopyThreads) copy_blocks_kernel(
    const CopyLayers layers, const int64_t* __restrict__ pairs, int64_t num_blocks,
    int64_t block_vecs, unsigned int* err) {
  const int64_t src = __ldg(pairs + 2 * (int64_t)blockIdx.x);
  const int64_t dst = __ldg(pairs + 2 * (int64_t)blockIdx.x + 1);
  if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) {
    if (threadIdx.x == 0 && blockIdx.y == 0) report(err, VFL_DEVERR_BLOCK_ID);
    return;
  }
  const int l = blockIdx.y >> 1;
  uint4* base = (blockIdx.y & 1) ? layers.v[l] : layers.k[l];
  const uint4* s = base + src * block_vecs;
  uint4* d = base + dst * block_vecs;
  for (int64_t i0 = threadIdx.x; i0 < block_vecs; i0 += kCopyThreads * kCopyUnroll) {
    uint4 v[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int64_t i = i0 + u * kCopyThreads;
      if (i < block_vecs) v[u] = ldg_nc_v4(s + i);
    }
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int64_t i = i0 + u * kCopyThreads;
      if (i < block_vecs) d[i] = v[u];
    }
  }
}

__global__ void prepare_decode_kernel(const int32_t* __restrict__ table, int64_t table_stride,
                                      int32_t table_cols, const int32_t* __restrict__ positions,
                                      int num_seqs, int block_size, int64_t* slot_mapping,
                                      int32_t* context_lens, int32_t* query_start_loc,
                                      unsigned int* err) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b > num_seqs) return;
  if (query_start_loc != nullptr) query_start_loc[b] = b;
  if (b == num_seqs) return;
  const int32_t pos = positions[b];
  const int32_t col = pos / block_size;
  if (pos < 0) {  // padding row of a fixed-size batch: nothing to append, nothing to attend
    if (context_lens != nullptr) context_lens[b] = 0;
    if (slot_mapping != nullptr) slot_mapping[b] = -1;
    return;
  }
  if (context_lens != nullptr) context_lens[b] = pos + 1;
  if (slot_mapping != nullptr) {
    if (col >= table_cols) {
      report(err, VFL_DEVERR_CONTEXT);
      slot_mapping[b] = -1;  // the append then skips this token
    } else {
      slot_mapping[b] = (int64_t)table[b * table_stride + col] * block_size + pos % block_size;
    }
  }
}

__global__ void paged_slots_kernel(const int32_t* __restrict__ pages, int64_t pages_stride,
                                   int32_t pages_cols, int num_reqs, int seq_len, int block_size,
                                   int64_t* slot_mapping, unsigned int* err) {
  const int64_t total = (int64_t)num_reqs * seq_len;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = i / seq_len;
    const int t = static_cast<int>(i - g * seq_len);
    const int col = t / block_size;
    if (col >= pages_cols) {
      if (t % block_size == 0) report(err, VFL_DEVERR_CONTEXT);
      slot_mapping[i] = -1;
      continue;
    }
    slot_mapping[i] = (int64_t)pages[g * pages_stride + col] * block_size + t % block_size;
  }
}

int grid_for(int64_t work_items, int threads) {
  const int64_t want = ceil_div(work_items, (int64_t)threads);
  const int64_t cap = (int64_t)kNumSMs * 16;  // grid-stride beyond 16 CTAs per SM
  return static_cast<int>(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace
}  // namespace vfl

using namespace vfl;

extern "C" {

int vfl_reshape_and_cache(const void* key, const void* value, void* k_cache, void* v_cache,
                          const int64_t* slot_mapping, int64_t num_tokens, int num_heads,
                          int head_dim, int block_size, int64_t num_blocks,
                          int64_t key_token_stride, int64_t value_token_stride, int dtype,
                          void* stream) {
  if (!dtype_ok(dtype)) return fail(VFL_ERR_UNSUPPORTED, "reshape_and_cache: dtype %d", dtype);
  if (num_tokens < 0 || num_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks <= 0)
    return fail(VFL_ERR_INVALID_ARGUMENT,
                "reshape_and_cache: bad sizes (tokens %lld, heads %d, head_dim %d, block_size %d, "
                "blocks %lld)",
                (long long)num_tokens, num_heads, head_dim, block_size, (long long)num_blocks);
  if (num_tokens == 0) return VFL_OK;
  const int64_t es = static_cast<int64_t>(dtype_size(dtype));
  const int64_t row_bytes = head_dim * es;
  if (row_bytes % 16 != 0)
    return fail(VFL_ERR_UNSUPPORTED, "reshape_and_cache: head_dim * element size must be a multiple of 16 bytes");
  if (!key || !value || !k_cache || !v_cache || !slot_mapping)
    return fail(VFL_ERR_INVALID_ARGUMENT, "reshape_and_cache: NULL pointer");
  if (!aligned16(key) || !aligned16(value) || !aligned16(k_cache) || !aligned16(v_cache) ||
      (key_token_stride * es) % 16 != 0 || (value_token_stride * es) % 16 != 0)
    return fail(VFL_ERR_INVALID_ARGUMENT, "reshape_and_cache: tensors and token strides must be 16-byte aligned");
  if (key_token_stride < num_heads * head_dim || value_token_stride < num_heads * head_dim)
    return fail(VFL_ERR_INVALID_ARGUMENT, "reshape_and_cache: token stride smaller than a token");
  unsigned int* err = nullptr;
  int st = device_error_word(&err);
  if (st) return st;
  const int row_vecs = static_cast<int>(row_bytes / 16);
  const int64_t work = num_tokens * num_heads * row_vecs;
  reshape_and_cache_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(key), static_cast<const uint8_t*>(value),
      static_cast<uint4*>(k_cache), static_cast<uint4*>(v_cache), slot_mapping, num_tokens,
      num_heads, row_vecs, block_size, num_blocks, key_token_stride * es, value_token_stride * es,
      err);
  return cuda_status(cudaGetLastError(), "reshape_and_cache launch");
}

int vfl_copy_blocks(void* const* k_caches, void* const* v_caches, int num_layers,
                    const int64_t* block_pairs, int num_pairs, int64_t num_blocks,
                    int64_t block_bytes, void* stream) {
  if (num_pairs < 0 || num_layers < 0 || num_blocks <= 0 || block_bytes <= 0)
    return fail(VFL_ERR_INVALID_ARGUMENT, "copy_blocks: bad sizes");
  if (num_pairs == 0 || num_layers == 0) return VFL_OK;
  if (num_layers > VFL_MAX_COPY_LAYERS)
    return fail(VFL_ERR_UNSUPPORTED, "copy_blocks: %d layers (at most %d per call)", num_layers,
                VFL_MAX_COPY_LAYERS);
  if (block_bytes % 16 != 0) return fail(VFL_ERR_INVALID_ARGUMENT, "copy_blocks: block_bytes % 16 != 0");
  if (!k_caches || !v_caches || !block_pairs) return fail(VFL_ERR_INVALID_ARGUMENT, "copy_blocks: NULL pointer");
  CopyLayers layers{};
  for (int l = 0; l < num_layers; ++l) {
    if (!k_caches[l] || !v_caches[l] || !aligned16(k_caches[l]) || !aligned16(v_caches[l]))
      return fail(VFL_ERR_INVALID_ARGUMENT, "copy_blocks: layer %d cache NULL or not 16-byte aligned", l);
    layers.k[l] = static_cast<uint4*>(k_caches[l]);
    layers.v[l] = static_cast<uint4*>(v_caches[l]);
  }
  unsigned int* err = nullptr;
  int st = device_error_word(&err);
  if (st) return st;
  dim3 grid(num_pairs, 2 * num_layers);
  copy_blocks_kernel<<<grid, kCopyThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      layers, block_pairs, num_blocks, block_bytes / 16, err);
  return cuda_status(cudaGetLastError(), "copy_blocks launch");
}

int vfl_prepare_decode(const int32_t* block_table, int64_t table_stride, int32_t table_cols,
                       const int32_t* positions, int num_seqs, int block_size,
                       int64_t* slot_mapping, int32_t* context_lens, int32_t* query_start_loc,
                       void* stream) {
  if (num_seqs < 0 || block_size <= 0 || table_cols < 0 || table_stride < table_cols)
    return fail(VFL_ERR_INVALID_ARGUMENT, "prepare_decode: bad sizes");
  if (num_seqs > 0 && (!positions || (slot_mapping && !block_table)))
    return fail(VFL_ERR_INVALID_ARGUMENT, "prepare_decode: NULL pointer");
  unsigned int* err = nullptr;
  int st = device_error_word(&err);
  if (st) return st;
  const int threads = 256;
  prepare_decode_kernel<<<ceil_div(num_seqs + 1, threads), threads, 0,
                          static_cast<cudaStream_t>(stream)>>>(
      block_table, table_stride, table_cols, positions, num_seqs, block_size, slot_mapping,
      context_lens, query_start_loc, err);
  return cuda_status(cudaGetLastError(), "prepare_decode launch");
}

int vfl_paged_slots(const int32_t* pages, int64_t pages_stride, int32_t pages_cols,
                    int num_reqs, int seq_len, int block_size, int64_t* slot_mapping,
                    void* stream) {
  if (num_reqs < 0 || seq_len < 0 || block_size <= 0 || pages_cols < 0 || pages_stride < pages_cols)
    return fail(VFL_ERR_INVALID_ARGUMENT, "paged_slots: bad sizes");
  if ((int64_t)num_reqs * seq_len == 0) return VFL_OK;
  if (!pages || !slot_mapping) return fail(VFL_ERR_INVALID_ARGUMENT, "paged_slots: NULL pointer");
  unsigned int* err = nullptr;
  int st = device_error_word(&err);
  if (st) return st;
  const int64_t work = (int64_t)num_reqs * seq_len;
  paged_slots_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      pages, pages_stride, pages_cols, num_reqs, seq_len, block_size, slot_mapping, err);
  return cuda_status(cudaGetLastError(), "paged_slots launch");
}

}  // extern "C"
