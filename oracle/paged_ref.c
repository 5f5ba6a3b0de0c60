/*
 * ORACLE — test infrastructure only. Never linked into, loaded by or called from the product
 * path (vflorence_b200/). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * use it, as the checker.
 *
 * A plain-C restatement of what the vflorence engine asks of the external CPU kernel library
 * `vllm_cpu_attn` (git dependency ducviet00/vllm-cpu-attention, pinned at uv.lock:1091-1093,
 * commit 79b2eb02549b3e047bc80df51321bc7281f851c9; not vendored, not installable here), plus the
 * torch index ops the engine runs beside it. The arithmetic follows the semantics the call sites
 * require (paths inside the vflorence project):
 *
 *   oracle_reshape_and_cache      vflorence/layers/attention.py:55-57 (decode append) and
 *                                 vflorence/engine/model_runner.py:252-259 (encoder pages):
 *                                 cache[slot // bs, h, slot % bs, :] = kv[t, h, :]
 *   oracle_attention              vflorence/layers/attention.py:61-72 (self, causal=False with
 *                                 one query per sequence, see :59-60) and :98-109 (cross):
 *                                 out = softmax(scale * q K^T) V over the first seq_len paged
 *                                 tokens, fp32 accumulation, two-pass softmax
 *   oracle_copy_blocks            vflorence/engine/model_runner.py:162-167: index_select of the
 *                                 sources, then index_copy_ into the destinations
 *   oracle_prepare_decode         vflorence/engine/model_runner.py:290-306
 *   oracle_paged_slots            vflorence/engine/model_runner.py:240-242
 *
 * Pinning: the attention restatement is checked against float64 softmax attention computed by
 * torch on the same pages (tests/golden/attention_cases.npz) and, end to end, by running the
 * unmodified reference engine on it: its greedy and beam tokens equal HuggingFace
 * transformers' generate() (tests/golden/engine_trace.*, made by tests/golden/make_golden.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { ORACLE_F32 = 0, ORACLE_BF16 = 1 };

static size_t elem_size(int dtype) { return dtype == ORACLE_F32 ? 4u : 2u; }

static float bf16_bits_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* Round-to-nearest-even float -> bfloat16 (NaN stays a quiet NaN). */
static uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float load_elem(const void* base, int64_t idx, int dtype) {
  if (dtype == ORACLE_F32) return ((const float*)base)[idx];
  return bf16_bits_to_f32(((const uint16_t*)base)[idx]);
}

static void store_elem(void* base, int64_t idx, float v, int dtype) {
  if (dtype == ORACLE_F32)
    ((float*)base)[idx] = v;
  else
    ((uint16_t*)base)[idx] = f32_to_bf16_bits(v);
}

int oracle_version(void) { return 1; }

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Returns the number of skipped out-of-range slots (negative slots are skipped silently). */
int64_t oracle_reshape_and_cache(const void* key, const void* value, void* k_cache,
                                 void* v_cache, const int64_t* slot_mapping, int64_t num_tokens,
                                 int num_heads, int head_dim, int block_size,
                                 int64_t num_blocks, int64_t key_stride, int64_t value_stride,
                                 int dtype) {
  const size_t es = elem_size(dtype);
  const size_t row = (size_t)head_dim * es;
  int64_t bad = 0;
  for (int64_t t = 0; t < num_tokens; ++t) {
    const int64_t slot = slot_mapping[t];
    if (slot < 0) continue;
    if (slot >= num_blocks * block_size) {
      ++bad;
      continue;
    }
    const int64_t blk = slot / block_size, off = slot % block_size;
    for (int h = 0; h < num_heads; ++h) {
      const size_t dst = (size_t)(((blk * num_heads + h) * block_size + off)) * row;
      memcpy((char*)k_cache + dst, (const char*)key + ((size_t)t * key_stride + (size_t)h * head_dim) * es, row);
      memcpy((char*)v_cache + dst, (const char*)value + ((size_t)t * value_stride + (size_t)h * head_dim) * es, row);
    }
  }
  return bad;
}

/*
 * Paged attention. query/output rows are [token, head, dim] with the given token strides.
 * query_start_loc: num_reqs + 1 entries; seq_lens: num_reqs; block_table: [num_reqs, stride].
 * Returns the number of (row, head) pairs whose pages referenced an out-of-range block
 * (those rows are written as zeros).
 */
int64_t oracle_attention(const void* query, int64_t q_stride, const void* k_cache,
                         const void* v_cache, int64_t num_blocks, void* output,
                         int64_t out_stride, const int32_t* query_start_loc,
                         const int32_t* seq_lens, int num_reqs, const int32_t* block_table,
                         int64_t table_stride, int num_heads, int head_dim, int block_size,
                         float scale, int causal, int dtype, int num_threads) {
  int64_t bad = 0;
  const int64_t total = (int64_t)num_reqs * num_heads;
#ifdef _OPENMP
  if (num_threads <= 0) num_threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(num_threads) reduction(+ : bad)
#endif
  for (int64_t rh = 0; rh < total; ++rh) {
    const int r = (int)(rh / num_heads), h = (int)(rh % num_heads);
    const int q_begin = query_start_loc[r], q_end = query_start_loc[r + 1];
    const int n = seq_lens[r];
    float* scores = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    float* acc = (float*)malloc(sizeof(float) * (size_t)head_dim);
    for (int i = q_begin; i < q_end; ++i) {
      const int visible = causal ? n - (q_end - 1 - i) : n;
      const int64_t qrow = (int64_t)i * q_stride + (int64_t)h * head_dim;
      const int64_t orow = (int64_t)i * out_stride + (int64_t)h * head_dim;
      int row_bad = 0;
      if (visible <= 0) {
        for (int d = 0; d < head_dim; ++d) store_elem(output, orow + d, 0.0f, dtype);
        continue;
      }
      /* pass 1: scores and their maximum */
      float m = -INFINITY;
      for (int t = 0; t < visible; ++t) {
        const int32_t blk = block_table[(int64_t)r * table_stride + t / block_size];
        if (blk < 0 || blk >= num_blocks) {
          row_bad = 1;
          break;
        }
        const int64_t krow = (((int64_t)blk * num_heads + h) * block_size + t % block_size) * head_dim;
        float dot = 0.0f;
        for (int d = 0; d < head_dim; ++d)
          dot += load_elem(query, qrow + d, dtype) * load_elem(k_cache, krow + d, dtype);
        scores[t] = dot * scale;
        if (scores[t] > m) m = scores[t];
      }
      if (row_bad) {
        ++bad;
        for (int d = 0; d < head_dim; ++d) store_elem(output, orow + d, 0.0f, dtype);
        continue;
      }
      /* pass 2: exponentials, their sum and the weighted values */
      float sum = 0.0f;
      for (int d = 0; d < head_dim; ++d) acc[d] = 0.0f;
      for (int t = 0; t < visible; ++t) {
        const int32_t blk = block_table[(int64_t)r * table_stride + t / block_size];
        const int64_t vrow = (((int64_t)blk * num_heads + h) * block_size + t % block_size) * head_dim;
        const float p = expf(scores[t] - m);
        sum += p;
        for (int d = 0; d < head_dim; ++d) acc[d] += p * load_elem(v_cache, vrow + d, dtype);
      }
      const float inv = 1.0f / sum;
      for (int d = 0; d < head_dim; ++d) store_elem(output, orow + d, acc[d] * inv, dtype);
    }
    free(scores);
    free(acc);
  }
  return bad;
}

/*
 * For each layer: copies of the source blocks are taken first, then written to the
 * destinations (index_select followed by index_copy_). Returns the number of skipped
 * out-of-range pairs.
 */
int64_t oracle_copy_blocks(void* const* k_caches, void* const* v_caches, int num_layers,
                           const int64_t* pairs, int num_pairs, int64_t num_blocks,
                           int64_t block_bytes) {
  int64_t bad = 0;
  char* tmp = (char*)malloc((size_t)block_bytes * (size_t)(num_pairs > 0 ? num_pairs : 1));
  for (int l = 0; l < 2 * num_layers; ++l) {
    char* cache = (char*)(l < num_layers ? k_caches[l] : v_caches[l - num_layers]);
    for (int p = 0; p < num_pairs; ++p) {
      const int64_t src = pairs[2 * p];
      if (src >= 0 && src < num_blocks)
        memcpy(tmp + (size_t)p * block_bytes, cache + (size_t)src * block_bytes, (size_t)block_bytes);
    }
    for (int p = 0; p < num_pairs; ++p) {
      const int64_t src = pairs[2 * p], dst = pairs[2 * p + 1];
      if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) {
        if (l == 0) ++bad;
        continue;
      }
      memcpy(cache + (size_t)dst * block_bytes, tmp + (size_t)p * block_bytes, (size_t)block_bytes);
    }
  }
  free(tmp);
  return bad;
}

void oracle_prepare_decode(const int32_t* block_table, int64_t table_stride,
                           const int32_t* positions, int num_seqs, int block_size,
                           int64_t* slot_mapping, int32_t* context_lens,
                           int32_t* query_start_loc) {
  for (int b = 0; b < num_seqs; ++b) {
    const int32_t pos = positions[b];
    query_start_loc[b] = b;
    if (pos < 0) { /* padding row */
      slot_mapping[b] = -1;
      context_lens[b] = 0;
      continue;
    }
    slot_mapping[b] = (int64_t)block_table[(int64_t)b * table_stride + pos / block_size] * block_size + pos % block_size;
    context_lens[b] = pos + 1;
  }
  query_start_loc[num_seqs] = num_seqs;
}

void oracle_paged_slots(const int32_t* pages, int64_t pages_stride, int num_reqs, int seq_len,
                        int block_size, int64_t* slot_mapping) {
  for (int g = 0; g < num_reqs; ++g)
    for (int t = 0; t < seq_len; ++t)
      slot_mapping[(int64_t)g * seq_len + t] =
          (int64_t)pages[(int64_t)g * pages_stride + t / block_size] * block_size + t % block_size;
}
