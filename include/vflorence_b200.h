/*
 * vflorence_b200 C ABI: the paged-KV attention path of the vflorence engine on B200 (sm_100a).
 *
 * The reference engine reaches this path through four functions of the external CPU library
 * `vllm_cpu_attn` plus one torch index op; each entry point below replaces one of them and
 * names the reference call site it replaces (paths are inside the vflorence project).
 *
 * Conventions
 *   - Plain pointers and sizes only. Every `void* stream` is a cudaStream_t (NULL = legacy
 *     default stream). Device pointers must belong to the current CUDA device.
 *   - No entry point allocates device memory, synchronises the stream or keeps a pointer
 *     after it returns. Scratch space is passed in by the caller (`workspace`).
 *   - Every entry point returns a vfl_status. On failure nothing was launched and
 *     vfl_last_error_message() describes the problem (thread-local string).
 *   - Arguments are validated on the host before any launch. What the host cannot see
 *     (block ids, slots and context lengths stored in device memory) is bounds-checked by the
 *     kernels: an out-of-range value is skipped (never dereferenced) and sets a bit in the
 *     per-device error word read by vfl_read_device_errors().
 *   - Layouts:
 *       paged K/V pool  [num_blocks, num_heads, block_size, head_dim], contiguous
 *       query / output  [num_tokens, num_heads, head_dim], token stride given, head and
 *                       element strides dense (head stride = head_dim)
 *       block_table     int32 [num_seqs, table_stride >= table_cols]
 *       slot_mapping    int64 [num_tokens], slot = block * block_size + offset, < 0 = skip
 */
#ifndef VFLORENCE_B200_H_
#define VFLORENCE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VFL_ABI_VERSION 4

typedef enum vfl_status {
  VFL_OK = 0,
  VFL_ERR_INVALID_ARGUMENT = 1, /* shape, stride, alignment, dtype or range error */
  VFL_ERR_UNSUPPORTED = 2,      /* valid for the reference, not built here (e.g. head_dim) */
  VFL_ERR_WORKSPACE = 3,        /* workspace missing or smaller than the plan needs */
  VFL_ERR_CUDA = 4,             /* a CUDA runtime call failed (launch, attribute, copy) */
  VFL_ERR_CAPACITY = 5          /* a host pool is exhausted (KV blocks, hypothesis slots) */
} vfl_status;

typedef enum vfl_dtype {
  VFL_DTYPE_F32 = 0,  /* torch.float32  */
  VFL_DTYPE_BF16 = 1  /* torch.bfloat16 */
} vfl_dtype;

/* Bits of the per-device error word (set by kernels, read by vfl_read_device_errors). */
#define VFL_DEVERR_BLOCK_ID 0x1u  /* block table entry or copy pair outside [0, num_blocks) */
#define VFL_DEVERR_SLOT 0x2u      /* slot_mapping entry >= num_blocks * block_size          */
#define VFL_DEVERR_CONTEXT 0x4u   /* seq_len > table_cols * block_size, or position beyond
                                     the table; the length was clamped                      */
#define VFL_DEVERR_TIMEOUT 0x8u   /* a bounded wait on a shared-memory barrier gave up      */
#define VFL_DEVERR_QUERY 0x10u    /* query_start_loc not non-decreasing / beyond num_tokens  */

/* How a plan spreads the work over CTAs.
 * VFL_SCHEDULE_ITEMS: one CTA per (request, head group, query chunk, split-K range).
 * VFL_SCHEDULE_BALANCED (tensor-core kernel, at most 8 query rows per request and 2048
 *   requests, no row tables):
 *   one persistent wave of num_splits CTAs; the (request, head group) items' 16-token tiles
 *   are laid end to end and each CTA takes an equal run of them, cutting items where the runs
 *   end; a second launch merges the pieces of cut items. Chosen for calls that would fill the
 *   GPU's CTA slots unevenly. */
typedef enum vfl_attention_schedule {
  VFL_SCHEDULE_ITEMS = 0,
  VFL_SCHEDULE_BALANCED = 1
} vfl_attention_schedule;

/* Launch plan for vfl_attention_with_kv_cache. Built on the host from host-side lengths;
 * plays the role of vllm_cpu_attn's opaque scheduler metadata. */
typedef struct vfl_attention_plan {
  int64_t magic;            /* VFL_PLAN_MAGIC once filled by vfl_plan_attention          */
  int32_t num_reqs;         /* requests (rows of block_table, entries of seq_lens)       */
  int32_t num_heads;
  int32_t head_dim;
  int32_t block_size;
  int32_t dtype;            /* vfl_dtype                                                 */
  int32_t causal;
  int32_t total_q;          /* query rows = query_start_loc[num_reqs]                    */
  int32_t max_q_len;        /* longest request in query rows                             */
  int32_t max_seq_len;      /* longest request in cached tokens                          */
  int32_t heads_per_cta;    /* heads handled by one CTA (one warp each)                  */
  int32_t queries_per_cta;  /* query rows of one request handled together: 1 or 4 (CUDA-core
                               kernel), 8 (tensor-core kernel: bf16, head_dim 64)          */
  int32_t blocks_per_split; /* KV blocks per split-K work item (VFL_SCHEDULE_ITEMS)      */
  int32_t num_splits;       /* split-K partitions of the longest request                 */
  int32_t stages;           /* shared-memory pipeline depth (16-token K/V tiles)         */
  int32_t merge_in_kernel;  /* split partials merged by the last split CTA (1) or by a
                               separate combine launch (0)                              */
  int64_t workspace_bytes;  /* scratch the caller must pass (0 = none)                   */
  int32_t row_tables;       /* 1: block_table rows are query rows (vfl_plan_attention_row_tables) */
  int32_t schedule;         /* vfl_attention_schedule                                    */
  int32_t min_tiles;        /* VFL_SCHEDULE_BALANCED: fewest 16-token tiles per CTA      */
  int32_t balanced_ctas;    /* VFL_SCHEDULE_BALANCED: CTAs of the persistent grid        */
} vfl_attention_plan;

#define VFL_PLAN_MAGIC 0x31504c4656LL /* "VFLP1" */

/* ---- library ---------------------------------------------------------------------------- */

/* ABI version of the loaded library (VFL_ABI_VERSION at build time). */
int vfl_abi_version(void);

/* Static description of a status code. */
const char* vfl_status_string(int status);

/* Message of the last failing call on this host thread ("" if none). */
const char* vfl_last_error_message(void);

/* Read (and with clear != 0 reset) the current device's error word. Synchronises `stream`. */
int vfl_read_device_errors(unsigned int* bits, int clear, void* stream);

/* (new: failure detection, no reference counterpart - the reference's failure handling is
 * host-side, vflorence/engine/llm_engine.py:68-80.) Exercises the bounded shared-memory wait
 * every pipelined kernel uses: one CTA whose consumer warp waits on a barrier that the producer
 * warp arrives on only when producer_arrives != 0. Otherwise the wait gives up after limit_ns
 * (in (0, 2e9]; VFL_ERR_INVALID_ARGUMENT else), VFL_DEVERR_TIMEOUT is set in the device error
 * word and the kernel exits; the context stays usable. Asynchronous on `stream`. Note: while
 * VFL_DEVERR_TIMEOUT is set, attention launches exit at once - read and clear the word with
 * vfl_read_device_errors before further work. */
int vfl_check_bounded_wait(int producer_arrives, int64_t limit_ns, void* stream);

/* ---- the four vllm_cpu_attn functions -------------------------------------------------------
 * replaces vllm_cpu_attn.get_isa(dtype, block_size, head_dim)
 *   (vflorence/engine/model_runner.py:38). Writes "sm100" into buf. Fails with
 *   VFL_ERR_UNSUPPORTED for a dtype, block size or head_dim the kernels do not cover. */
int vfl_get_isa(int dtype, int block_size, int head_dim, char* buf, int buf_len);

/* replaces vllm_cpu_attn.get_scheduler_metadata(...)
 *   (vflorence/layers/attention.py:18-29, vflorence/engine/model_runner.py:308-319).
 * seq_lens_host / query_start_loc_host are HOST arrays of num_reqs / num_reqs + 1 entries;
 * query_start_loc_host may be NULL for one query row per request. */
int vfl_plan_attention(int num_reqs, int num_heads, int num_kv_heads, int head_dim,
                       int block_size, int dtype, int causal, const int32_t* seq_lens_host,
                       const int32_t* query_start_loc_host, vfl_attention_plan* plan);

/* A plan for requests whose query rows each have their own block table - the beams of one
 * request in beam search, which share most of their blocks (copy-on-write forks) but not all.
 * With this plan, vfl_attention_with_kv_cache reads row i's table at block_table + i *
 * table_stride (query rows, not requests); query_start_loc groups the rows of a request and
 * seq_lens holds one length per request (its rows must all see that many tokens). A CTA serves
 * up to 8 rows of a request and loads each distinct block of a tile position once, for all the
 * rows that hold it. Extends vllm_cpu_attn.get_scheduler_metadata (attention.py:18-29), where
 * every beam is its own request. bf16 with head_dim 64 only (VFL_ERR_UNSUPPORTED otherwise);
 * never causal. */
int vfl_plan_attention_row_tables(int num_reqs, int num_heads, int num_kv_heads, int head_dim,
                                  int block_size, int dtype, const int32_t* seq_lens_host,
                                  const int32_t* query_start_loc_host, vfl_attention_plan* plan);

/* (new: no reference counterpart - vllm_cpu_attn's metadata is opaque.) Re-plans `plan` (from
 * vfl_plan_attention) for the given vfl_attention_schedule: VFL_SCHEDULE_ITEMS, or
 * VFL_SCHEDULE_BALANCED with at least min_tiles 16-token tiles per CTA (0: the default).
 * Updates workspace_bytes; keeps the plan's stage count (the planner gives balanced plans two).
 * VFL_ERR_UNSUPPORTED when the plan cannot be balanced (not the
 * tensor-core kernel, row tables, more than 8 query rows per request, more than 2048 requests,
 * or a request of 2^24 tokens or more). */
int vfl_plan_attention_schedule(vfl_attention_plan* plan, int schedule, int min_tiles);

/* replaces vllm_cpu_attn.reshape_and_cache(key, value, k_cache, v_cache, slot_mapping, isa=)
 *   (vflorence/layers/attention.py:55-57, vflorence/engine/model_runner.py:252-259).
 * cache[slot // block_size, h, slot % block_size, :] = key[t, h, :] for every token t with
 * slot = slot_mapping[t] >= 0. key/value token strides are in elements. */
int vfl_reshape_and_cache(const void* key, const void* value, void* k_cache, void* v_cache,
                          const int64_t* slot_mapping, int64_t num_tokens, int num_heads,
                          int head_dim, int block_size, int64_t num_blocks,
                          int64_t key_token_stride, int64_t value_token_stride, int dtype,
                          void* stream);

/* replaces vllm_cpu_attn.attention_with_kv_cache(query, k_cache, v_cache, output,
 *   query_start_loc, seq_lens, scale=, causal=, block_table=, scheduler_metadata=)
 *   (vflorence/layers/attention.py:61-72 and :98-109).
 * For request r with query rows [query_start_loc[r], query_start_loc[r+1]) and n = seq_lens[r]
 * cached tokens, row i attends to the first n tokens (causal: n - (q_end - 1 - i)) of the
 * pages block_table[r, :]:  out = softmax(scale * q K^T) V, fp32 accumulation.
 * A request with no visible tokens produces zeros. Rows of several queries that share one
 * request (beams over one encoder) read each K/V page once. */
int vfl_attention_with_kv_cache(const vfl_attention_plan* plan, const void* query,
                                int64_t query_token_stride, const void* k_cache,
                                const void* v_cache, int64_t num_blocks, void* output,
                                int64_t output_token_stride, const int32_t* query_start_loc,
                                const int32_t* seq_lens, const int32_t* block_table,
                                int64_t table_stride, int32_t table_cols, float scale,
                                void* workspace, size_t workspace_bytes, void* stream);

/* replaces the two calls of the decoder's self-attention op, vllm_cpu_attn.reshape_and_cache
 *   then vllm_cpu_attn.attention_with_kv_cache (vflorence/layers/attention.py:55-72), with one
 *   launch: query row t brings one new token, key / value [num_heads, head_dim] dense at key +
 *   t * key_token_stride (elements), written to slot_mapping[t] (negative: none; past the pool:
 *   skipped and flagged VFL_DEVERR_SLOT) before the attention reads it. The token is the newest
 *   position of its sequence (seq_lens - 1), or for causal rows the successive positions ending
 *   there. Otherwise as vfl_attention_with_kv_cache; the slot's block must be the row's own (not
 *   shared with another row of the call, as after copy-on-write). Plans where
 *   vfl_attention_append_supported is 0 get VFL_ERR_UNSUPPORTED: then append, then attend. */
int vfl_attention_with_kv_cache_append(const vfl_attention_plan* plan, const void* query,
                                       int64_t query_token_stride, const void* key, int64_t key_token_stride,
                                       const void* value, int64_t value_token_stride,
                                       const int64_t* slot_mapping, const void* k_cache, const void* v_cache,
                                       int64_t num_blocks, void* output, int64_t output_token_stride,
                                       const int32_t* query_start_loc, const int32_t* seq_lens,
                                       const int32_t* block_table, int64_t table_stride, int32_t table_cols,
                                       float scale, void* workspace, size_t workspace_bytes, void* stream);

/* 1 when vfl_attention_with_kv_cache_append takes this plan: one new token per query row, and
 * either one row per request (every dtype and head_dim), or with the tensor-core kernel (bf16,
 * head_dim 64) causal rows, at most 8 per request (one CTA holds them all, since each row
 * reads the rows before it), or row tables. */
int vfl_attention_append_supported(const vfl_attention_plan* plan);

/* No counterpart in the reference (vllm_cpu_attn allocates on the host heap as it likes).
 * The same attention as vfl_attention_with_kv_cache, for callers that cannot allocate device
 * memory - a C/C++ or FFI host without a device allocator of its own, where every scratch
 * buffer would be a device-synchronising cudaMalloc, or a process whose device memory a
 * framework's pool already holds. Takes no workspace: the split-K scratch is a fixed array of
 * VFL_STATIC_WORKSPACE_BYTES inside the library, which every device that loads the library
 * keeps until exit. Plans needing more scratch fail with VFL_ERR_WORKSPACE. All calls on a
 * device share that array: calls that can overlap on the device race, so order them. Plans
 * from vfl_plan_attention keep no state in it between calls; a caller-built plan with
 * merge_in_kernel = 1 keeps arrival counters there, which such a call clears first. The first
 * call on a device looks up the array's address (cached for the process; not valid after
 * cudaDeviceReset); make it before any stream capture. */
#define VFL_STATIC_WORKSPACE_BYTES (64u * 1024u * 1024u)
int vfl_attention_with_kv_cache_no_alloc(const vfl_attention_plan* plan, const void* query,
                                         int64_t query_token_stride, const void* k_cache,
                                         const void* v_cache, int64_t num_blocks, void* output,
                                         int64_t output_token_stride,
                                         const int32_t* query_start_loc, const int32_t* seq_lens,
                                         const int32_t* block_table, int64_t table_stride,
                                         int32_t table_cols, float scale, void* stream);

/* ---- around the four ops --------------------------------------------------------------------
 * replaces ModelRunner._copy_blocks (vflorence/engine/model_runner.py:162-167):
 * for every layer l and pair p: k_caches[l][dst_p] = k_caches[l][src_p], same for v_caches,
 * with gather-then-scatter meaning (all sources are read before any destination is written
 * requires disjoint source and destination sets, which copy-on-write guarantees; the host
 * wrapper checks it). block_pairs: device int64 [num_pairs, 2] = (src, dst). block_bytes =
 * num_heads * block_size * head_dim * element size. One launch for all layers. */
#define VFL_MAX_COPY_LAYERS 128
int vfl_copy_blocks(void* const* k_caches, void* const* v_caches, int num_layers,
                    const int64_t* block_pairs, int num_pairs, int64_t num_blocks,
                    int64_t block_bytes, void* stream);

/* replaces the per-step list building of ModelRunner._prepare
 *   (vflorence/engine/model_runner.py:290-306) on the device: for sequence b at position
 *   p = positions[b] (= num_cached_tokens):
 *     slot_mapping[b] = block_table[b, p // block_size] * block_size + p % block_size
 *     context_lens[b] = p + 1
 *     query_start_loc[b] = b  (and query_start_loc[num_seqs] = num_seqs)
 *   A negative position marks a padding row (fixed-size batches): slot -1, context length 0.
 *   Any output pointer may be NULL. */
int vfl_prepare_decode(const int32_t* block_table, int64_t table_stride, int32_t table_cols,
                       const int32_t* positions, int num_seqs, int block_size,
                       int64_t* slot_mapping, int32_t* context_lens, int32_t* query_start_loc,
                       void* stream);

/* replaces the encoder K/V projection and page write of ModelRunner._encode
 *   (vflorence/engine/model_runner.py:248-259: per layer kv_proj, then reshape_and_cache) with
 *   one tensor-core launch per layer: kv = hidden . w_kv^T (+ bias) with fp32 accumulation,
 *   token t's k half written to k_cache[slot // block_size, h, slot % block_size, :] and its v
 *   half to v_cache likewise (slot = slot_mapping[t]; negative slots skipped, slots past the pool
 *   flagged with VFL_DEVERR_SLOT). bf16 only. hidden: [num_tokens, hidden_dim] with rows
 *   hidden_stride elements apart; w_kv: [2 * num_heads * head_dim, hidden_dim] row-major (a
 *   torch.nn.Linear weight holding the k rows, then the v rows); bias: [2 * num_heads *
 *   head_dim] or NULL. hidden_dim a multiple of 64, head_dim of 32, 2 * num_heads * head_dim
 *   of 128 (VFL_ERR_UNSUPPORTED otherwise); 16-byte aligned pointers and row stride. */
int vfl_kv_proj_paged(const void* hidden, int64_t hidden_stride, const void* w_kv, const void* bias,
                      void* k_cache, void* v_cache, const int64_t* slot_mapping, int64_t num_tokens,
                      int32_t hidden_dim, int32_t num_heads, int32_t head_dim, int32_t block_size,
                      int64_t num_blocks, void* stream);

/* replaces the post-norm residual of the decoder that calls the paged ops
 *   (vflorence/models/bart.py:192-201, LayerNorm(hidden + sublayer(hidden)) after the
 *   self-attention, the cross-attention and the FFN; and bart.py:260-264, the embedding's
 *   LayerNorm(tokens + positions)): out = LayerNorm(h + x) * weight + bias over rows of
 *   hidden_dim elements, in one launch. h + x is rounded to dtype first, as a separate add does;
 *   mean and biased variance in fp32; eps as torch.nn.LayerNorm. bias may be NULL. Strides are
 *   in elements; pointers and strides 16-byte aligned. hidden_dim must satisfy
 *   vfl_add_layernorm_supported (a multiple of 256 elements up to 2048 for bf16, of 128 up to
 *   1024 for fp32), VFL_ERR_UNSUPPORTED otherwise. out may alias h or x. */
int vfl_add_layernorm(const void* h, int64_t h_stride, const void* x, int64_t x_stride,
                      const void* weight, const void* bias, void* out, int64_t out_stride,
                      int32_t rows, int32_t hidden_dim, float eps, int32_t dtype, void* stream);

/* 1 when vfl_add_layernorm is built for this dtype and hidden_dim, else 0. */
int vfl_add_layernorm_supported(int dtype, int hidden_dim);

/* Activations fused into vfl_decode_linear. */
#define VFL_ACT_NONE 0
#define VFL_ACT_GELU 1 /* exact: 0.5 x (1 + erf(x / sqrt 2)), transformers' "gelu" */

/* replaces, for decode steps of at most 16 rows, the decoder's linear layers
 *   (vflorence/models/bart.py:106-146: q/k/v, out, cross q/out, fc1 + activation, fc2) and the
 *   vocabulary projection (bart.py:311-316), which the reference runs as torch GEMMs:
 *   y[m, n] = act(sum_k x[m, k] * weight[n, k] + bias[n]) for m < rows, n < n, with weight
 *   [n, k] row-major (torch.nn.Linear's layout). float32. One launch; a K split runs in a thread-
 *   block cluster whose partial sums are added in a fixed order (results do not depend on
 *   timing). Strides in elements; x, weight, y 16-byte aligned, x_stride a multiple of 4;
 *   bias may be NULL. VFL_ERR_UNSUPPORTED unless vfl_decode_linear_supported. */
int vfl_decode_linear(const void* x, int64_t x_stride, const void* weight, const void* bias, void* y,
                      int64_t y_stride, int32_t rows, int32_t n, int32_t k, int32_t dtype,
                      int32_t activation, void* stream);

/* 1 when vfl_decode_linear is built for this shape: float32, 1 <= rows <= 16, n a multiple of
 * 32, k a multiple of 128 (with each K slice of the rows fitting 64 KiB of shared memory). */
int vfl_decode_linear_supported(int dtype, int rows, int n, int k);

/* replaces the encoder slot computation of ModelRunner._encode
 *   (vflorence/engine/model_runner.py:240-242): for request g and token t < seq_len,
 *   slot_mapping[g * seq_len + t] = pages[g, t // block_size] * block_size + t % block_size. */
int vfl_paged_slots(const int32_t* pages, int64_t pages_stride, int32_t pages_cols,
                    int num_reqs, int seq_len, int block_size, int64_t* slot_mapping,
                    void* stream);

/* ---- candidate selection of a decode step ----------------------------------------------------
 * replaces, on the device, the float copy, log_softmax, top-k and cumulative-log-prob add of
 *   ModelRunner._sample / _beam_search (vflorence/engine/model_runner.py:370-371, :394-399)
 *   and the greedy argmax (:379-380). Row r of `scores` (float32 or bfloat16, `vocab` entries at
 *   `row_stride` elements apart) gives its best k entries:
 *     value = log_softmax ? (x - max_r) - log(sum_v exp(x_v - max_r)) : x, plus row_offset[r]
 *             when row_offset is not NULL (float32, device)
 *   ordered by value descending, equal values by lower index (the argmax rule; the reference's
 *   CPU top-k leaves that order unspecified). values: float32 [rows, k]; indices: int32
 *   [rows, k]. k in [1, 64] and <= vocab. With log_softmax the entries are chosen on x, which
 *   log_softmax maps monotonically. */
int vfl_row_topk(const void* scores, int32_t dtype, int64_t rows, int64_t vocab, int64_t row_stride,
                 int32_t log_softmax, const float* row_offset, int32_t k, float* values,
                 int32_t* indices, void* workspace, size_t workspace_bytes, void* stream);

/* Scratch vfl_row_topk needs for `rows` x `vocab` at this k: 0, or the bytes of the per-chunk
 * partial results when rows are split across several CTAs (16-byte aligned, no initial
 * contents needed). VFL_ERR_WORKSPACE when a call gets less. */
size_t vfl_row_topk_workspace_size(int64_t rows, int64_t vocab, int32_t k);

/* replaces the per-request merge of ModelRunner._beam_search (model_runner.py:401-410): the
 *   rows of request group g (groups[r] == g, at most 64 rows, placed by ranks[r]) pool their
 *   k candidates from vfl_row_topk, ordered by value descending, equal values in row-rank then
 *   list order (a stable sort of the rows' lists in row order); the best `keep` are written to
 *   out, int32 [3, num_groups, keep]: row, token index, float32 bits of the value; row -1 pads
 *   a group with fewer than `keep` candidates. All pointers are device pointers. */
int vfl_beam_merge(const float* values, const int32_t* indices, int64_t rows, int32_t k,
                   const int32_t* groups, const int32_t* ranks, int32_t num_groups, int32_t keep,
                   int32_t* out, void* stream);

/* replaces Sequence.fork's child.token_ids = [*parent.token_ids, token]
 *   (vflorence/engine/sequence.py:53-55) for the device token rows of a beam step: for each
 *   born child i, tokens[child_i, :width] = tokens[parent_i, :width] with tokens[child_i, pos_i]
 *   = token_i. born: device int32 [4, num_born] (parents, children, positions, tokens). No child
 *   may be a parent of the same call (the decode runtime's slots never are). Rows out of range
 *   or a position past width are skipped and flagged with VFL_DEVERR_SLOT. */
int vfl_fork_token_rows(int32_t* tokens, int64_t row_stride, int32_t num_rows, int32_t width,
                        const int32_t* born, int32_t num_born, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VFLORENCE_B200_H_ */
