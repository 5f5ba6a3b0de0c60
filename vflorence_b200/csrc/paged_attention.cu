// Planner and C-ABI launcher for the paged attention kernels.
//
// vfl_plan_attention plays the part of vllm_cpu_attn.get_scheduler_metadata
// (vflorence/layers/attention.py:18-29, vflorence/engine/model_runner.py:308-319): from the
// host-side lengths it fixes the CTA shape, the shared-memory pipeline depth and the split-K
// partition, and the workspace those splits need. It is pure host arithmetic (no CUDA call),
// sized for B200's 148 SMs.
#include <cmath>
#include <mutex>

#include "paged_attention_kernels.cuh"

namespace vfl {
namespace {

// split-K rule thresholds, in tokens (measured on B200; see the split rule in vfl_plan_attention)
constexpr int kNoSplitTokens = 128;     // contexts this short never split
constexpr int kMinSplitTokens = 96;     // a split that fills the GPU keeps at least this many tokens
constexpr int kLongSplitTokens = 512;   // ... and no split of a near-uniform batch holds more
constexpr int kSkewSplitTokens = 320;   // skewed lengths (max > 1.5 x mean): pieces of at least this
constexpr int kShortItemTokens = 256;   // items this short run 2-stage rings when they fill a wave
constexpr int kSmemPerSM = 227 * 1024;

int plan_fail(vfl_attention_plan* plan, int status) {
  if (plan) plan->magic = 0;
  return status;
}

// The tensor-core kernel covers bfloat16 pools with head_dim 64 (the BART / Florence-2 shape).
bool use_tensor_cores(int dtype, int head_dim) { return dtype == VFL_DTYPE_BF16 && head_dim == 64; }

// ---- TMA tensor maps of the K/V pools (driver entry point through the runtime; cached)
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct MapEntry {
  const void* base;
  uint64_t rows;
  uint32_t box_rows;
  CUtensorMap map;
};
constexpr int kMapCache = 32;
MapEntry g_maps[kMapCache];
int g_map_next = 0;
std::mutex g_map_mutex;

int encode_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  if (fn == nullptr)
    return fail(VFL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorString(err));
  *out = fn;
  return VFL_OK;
}

// [rows, 64] bf16 pool, 128-byte swizzle, box 64 x box_rows.
int pool_tensor_map(const void* base, uint64_t rows, uint32_t box_rows, CUtensorMap* out) {
  std::lock_guard<std::mutex> lock(g_map_mutex);
  for (const MapEntry& e : g_maps)
    if (e.base == base && e.rows == rows && e.box_rows == box_rows) {
      *out = e.map;
      return VFL_OK;
    }
  EncodeTiledFn fn = nullptr;
  int st = encode_fn(&fn);
  if (st) return st;
  CUtensorMap map;
  const cuuint64_t dims[2] = {64, rows};
  const cuuint64_t strides[1] = {64 * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t elem_strides[2] = {1, 1};
  const CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                        elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VFL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  g_maps[g_map_next] = MapEntry{base, rows, box_rows, map};
  g_map_next = (g_map_next + 1) % kMapCache;
  *out = map;
  return VFL_OK;
}

}  // namespace

// A row-major bf16 matrix [outer rows, inner columns] (rows `row_bytes` apart) as a 2-D tensor
// map with the 128-byte swizzle, box inner x outer; reads outside the matrix fill zeros.
int make_tensor_map_2d_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                            uint32_t box_outer, CUtensorMap* out) {
  EncodeTiledFn fn = nullptr;
  int st = encode_fn(&fn);
  if (st) return st;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem_strides[2] = {1, 1};
  const CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                        elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VFL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VFL_OK;
}

// The balanced schedule's shapes: the tensor-core kernel, one query chunk per request, one
// block table per request, lengths and rows that fit its shared-memory arrays.
bool balanced_supported(const vfl_attention_plan* plan) {
  return plan->queries_per_cta == kTcRows && use_tensor_cores(plan->dtype, plan->head_dim) && plan->row_tables == 0 &&
         plan->max_q_len <= kTcRows && plan->num_reqs >= 1 && plan->num_reqs <= kBalancedMaxReqs &&
         plan->max_seq_len < kBalancedMaxLen;
}

// Workspace of an item-schedule plan: acc partials | (m, l) partials | arrival counters.
int64_t items_workspace(const vfl_attention_plan* plan) {
  if (plan->num_splits <= 1) return 0;
  const int64_t items = (int64_t)plan->total_q * plan->num_heads * plan->num_splits;
  const int64_t q_chunks =
      ceil_div((int64_t)(plan->max_q_len < 1 ? 1 : plan->max_q_len), (int64_t)plan->queries_per_cta);
  return ceil_div(items * plan->head_dim * 4, (int64_t)256) * 256 + ceil_div(items * 2 * 4, (int64_t)256) * 256 +
         (plan->merge_in_kernel
              ? (int64_t)plan->num_reqs * (plan->num_heads / plan->heads_per_cta) * q_chunks * 4
              : 0);
}

// Sets a plan's schedule and the fields and workspace it implies (the plan is otherwise filled).
int set_schedule(vfl_attention_plan* plan, int schedule, int min_tiles) {
  if (schedule == VFL_SCHEDULE_ITEMS) {
    plan->schedule = VFL_SCHEDULE_ITEMS;
    plan->min_tiles = 0;
    plan->balanced_ctas = 0;
    plan->workspace_bytes = items_workspace(plan);
    return VFL_OK;
  }
  if (schedule != VFL_SCHEDULE_BALANCED)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: schedule %d", schedule);
  if (!balanced_supported(plan))
    return fail(VFL_ERR_UNSUPPORTED,
                "attention: the balanced schedule needs bf16 with head_dim 64, one block table per request, "
                "at most %d query rows per request, %d requests and %d tokens per request",
                kTcRows, kBalancedMaxReqs, kBalancedMaxLen - 1);
  if (min_tiles < 0) return fail(VFL_ERR_INVALID_ARGUMENT, "attention: min_tiles %d < 0", min_tiles);
  const int hpc = plan->heads_per_cta;
  const int stage_bytes = 2 * hpc * 16 * plan->head_dim * 2;
  const int smem = kTcHeaderBytes + plan->stages * stage_bytes + balanced_sched_bytes(plan->num_reqs);
  int per_sm = kSmemPerSM / (smem + 1024);
  per_sm = per_sm > kBalancedCtasPerSM ? kBalancedCtasPerSM : per_sm;
  if (per_sm < 1) return fail(VFL_ERR_UNSUPPORTED, "attention: balanced ring of %d stages too large", plan->stages);
  plan->schedule = VFL_SCHEDULE_BALANCED;
  plan->min_tiles = min_tiles > 0 ? min_tiles : kBalancedMinTiles;
  plan->balanced_ctas = kNumSMs * per_sm;
  plan->workspace_bytes = BalancedWorkspace(plan->balanced_ctas, hpc, plan->num_reqs, plan->num_heads).total();
  return VFL_OK;
}

// Whether the balanced schedule beats the item grid for a plan (rule fitted below).
// Whether the balanced schedule beats the item grid: `work` 16-token tiles over `items`
// (request, head group) items, which the grid runs as `grid_ctas` CTAs (`splits` split-K
// pieces of the longest request). Fitted to device time on B200 with L2 flushed (bf16, 16 heads
// x 64, block 16; 8-1024 requests x 1, 3 or 4 rows x 128-4096 tokens, near-uniform U[3/4 ctx,
// ctx] and skewed U[1, ctx] lengths; 132 shapes):
//   * a grid of at most one wave (148 SMs x 3 CTAs) runs all its CTAs at once and pays no
//     pieces to merge: the grid wins or ties (the balanced wave: 0.65-1.06 x);
//   * items of fewer than 16 tiles on average: the balanced wave's fixed cost (the length scan,
//     the merge launch) outweighs its gain (0.89-1.05 x);
//   * near-uniform lengths that the grid runs unsplit in four waves or more are already even
//     (0.986-1.0 x);
//   * otherwise the balanced wave wins, by 0.997-1.38 x (1.04 x at 1024 requests of U[1, 4096]
//     tokens; most where lengths are skewed, or a split grid lands between whole waves).
bool balanced_pays_off(const vfl_attention_plan* plan, int64_t work, int64_t items, int64_t grid_ctas, int64_t splits,
                       bool skewed) {
  if (!balanced_supported(plan) || items <= 0) return false;
  const int64_t wave = (int64_t)kNumSMs * kBalancedCtasPerSM;
  if (grid_ctas <= wave || work < 16 * items) return false;
  if (!skewed && splits == 1 && grid_ctas >= 4 * wave) return false;
  return true;
}

// A plan is caller memory: every constraint the kernels rely on (shared-memory table slice,
// stage ring, CTA shape, workspace size) is re-derived here before anything touches the device.
int check_attention_plan(const vfl_attention_plan* plan) {
  const int H = plan->num_heads, D = plan->head_dim, bs = plan->block_size;
  if (plan->num_reqs < 0 || plan->total_q < 0 || plan->total_q > INT32_MAX / 2 || plan->max_q_len < 0 ||
      plan->max_seq_len < 0 || H <= 0 || (plan->causal != 0 && plan->causal != 1))
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan counts out of range");
  if (!dtype_ok(plan->dtype) || !head_dim_supported(D) || bs < 16 || bs > 1024 || bs % 16 != 0)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan dtype / head_dim / block_size not built");
  const int hpc = plan->heads_per_cta, qpc = plan->queries_per_cta;
  if (!(hpc == 1 || hpc == 2 || hpc == 4) || H % hpc != 0)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan heads_per_cta %d for %d heads", hpc, H);
  const bool tc = qpc == kTcRows;
  if (tc ? !use_tensor_cores(plan->dtype, D) : !(qpc == 1 || qpc == 4))
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan queries_per_cta %d not built for this shape", qpc);
  if (plan->stages < 2 || plan->stages > kMaxStages)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan stages %d outside [2, %d]", plan->stages, kMaxStages);
  const int64_t stage_bytes = (int64_t)2 * hpc * 16 * D * (int64_t)dtype_size(plan->dtype);
  if ((tc ? kTcHeaderBytes : kHeaderBytes) + plan->stages * stage_bytes > 227 * 1024)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan stages do not fit in shared memory");
  if (plan->blocks_per_split < 1 || plan->blocks_per_split > kMaxBlocksPerSplit || plan->num_splits < 1 ||
      plan->num_splits > 65535)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan split %d x %d blocks outside [1, 65535] x [1, %d]",
                plan->num_splits, plan->blocks_per_split, kMaxBlocksPerSplit);
  const int64_t max_blocks = ceil_div((int64_t)plan->max_seq_len, (int64_t)bs);
  if ((int64_t)plan->num_splits * plan->blocks_per_split < max_blocks)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan splits do not cover max_seq_len %d", plan->max_seq_len);
  if (plan->merge_in_kernel != 0 && plan->merge_in_kernel != 1)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan merge mode %d", plan->merge_in_kernel);
  if (plan->row_tables != 0 && (plan->row_tables != 1 || !tc || plan->causal))
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan row_tables needs the tensor-core kernel, not causal");
  if (plan->schedule != VFL_SCHEDULE_ITEMS && plan->schedule != VFL_SCHEDULE_BALANCED)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan schedule %d", plan->schedule);
  if (plan->schedule == VFL_SCHEDULE_BALANCED) {
    if (!balanced_supported(plan))
      return fail(VFL_ERR_INVALID_ARGUMENT, "attention: balanced plan outside the balanced kernel's shapes");
    if (plan->min_tiles < 1 || plan->balanced_ctas < 1 || plan->balanced_ctas > kNumSMs * kBalancedCtasPerSM)
      return fail(VFL_ERR_INVALID_ARGUMENT, "attention: balanced plan min_tiles %d / %d CTAs", plan->min_tiles,
                  plan->balanced_ctas);
    if (kTcHeaderBytes + plan->stages * stage_bytes + balanced_sched_bytes(plan->num_reqs) > 227 * 1024)
      return fail(VFL_ERR_INVALID_ARGUMENT, "attention: balanced plan does not fit in shared memory");
    const int64_t need = BalancedWorkspace(plan->balanced_ctas, hpc, plan->num_reqs, H).total();
    if (plan->workspace_bytes < need)
      return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan workspace_bytes %lld < the %lld its schedule needs",
                  (long long)plan->workspace_bytes, (long long)need);
    return VFL_OK;
  }
  const int64_t q_chunks = ceil_div((int64_t)(plan->max_q_len < 1 ? 1 : plan->max_q_len), (int64_t)qpc);
  if (q_chunks > 65535 || (int64_t)plan->num_reqs * (H / hpc) > INT32_MAX)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan launch grid too large");
  if (plan->num_splits > 1) {
    const int64_t items = (int64_t)plan->total_q * H * plan->num_splits;
    const int64_t need = ceil_div(items * D * 4, (int64_t)256) * 256 + ceil_div(items * 2 * 4, (int64_t)256) * 256 +
                         (plan->merge_in_kernel ? (int64_t)plan->num_reqs * (H / hpc) * q_chunks * 4 : 0);
    if (plan->workspace_bytes < need)
      return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan workspace_bytes %lld < the %lld its splits need",
                  (long long)plan->workspace_bytes, (long long)need);
  }
  return VFL_OK;
}

}  // namespace vfl

using namespace vfl;

extern "C" {

int vfl_plan_attention(int num_reqs, int num_heads, int num_kv_heads, int head_dim, int block_size,
                       int dtype, int causal, const int32_t* seq_lens_host,
                       const int32_t* query_start_loc_host, vfl_attention_plan* plan) {
  if (plan == nullptr) return fail(VFL_ERR_INVALID_ARGUMENT, "plan is NULL");
  if (num_reqs < 0 || num_heads <= 0)
    return plan_fail(plan, fail(VFL_ERR_INVALID_ARGUMENT, "num_reqs %d / num_heads %d", num_reqs, num_heads));
  if (num_kv_heads != num_heads)
    return plan_fail(plan, fail(VFL_ERR_UNSUPPORTED,
                                "num_kv_heads %d != num_heads %d: grouped-query attention is not built "
                                "(the engine's BART/Florence-2 decoders are multi-head)",
                                num_kv_heads, num_heads));
  char isa[8];
  int st = vfl_get_isa(dtype, block_size, head_dim, isa, sizeof(isa));
  if (st) return plan_fail(plan, st);
  if (num_reqs > 0 && seq_lens_host == nullptr)
    return plan_fail(plan, fail(VFL_ERR_INVALID_ARGUMENT, "seq_lens_host is NULL"));

  int64_t total_q = 0, max_q = 0, max_seq = 0;
  if (query_start_loc_host && query_start_loc_host[0] < 0)
    return plan_fail(plan, fail(VFL_ERR_INVALID_ARGUMENT, "query_start_loc[0] < 0"));
  for (int r = 0; r < num_reqs; ++r) {
    const int64_t n = seq_lens_host[r];
    if (n < 0) return plan_fail(plan, fail(VFL_ERR_INVALID_ARGUMENT, "seq_lens[%d] = %lld < 0", r, (long long)n));
    const int64_t ql = query_start_loc_host ? (int64_t)query_start_loc_host[r + 1] - query_start_loc_host[r] : 1;
    if (ql < 0)
      return plan_fail(plan, fail(VFL_ERR_INVALID_ARGUMENT, "query_start_loc decreases at %d", r));
    max_q = ql > max_q ? ql : max_q;
    max_seq = n > max_seq ? n : max_seq;
  }
  total_q = num_reqs == 0 ? 0 : (query_start_loc_host ? query_start_loc_host[num_reqs] : num_reqs);
  if (total_q > INT32_MAX / 2)
    return plan_fail(plan, fail(VFL_ERR_UNSUPPORTED, "too many query rows (%lld)", (long long)total_q));

  const int es = static_cast<int>(dtype_size(dtype));
  int hpc = 4;
  while (hpc > 1 && (num_heads % hpc != 0 || 2 * hpc * 16 * head_dim * es > 32 * 1024)) hpc >>= 1;
  const int stage_bytes = 2 * hpc * 16 * head_dim * es;
  int stages = kMaxStageBytes / stage_bytes;
  stages = stages < 2 ? 2 : (stages > 4 ? 4 : stages);
  const bool tc = use_tensor_cores(dtype, head_dim);
  const int qpc = tc ? kTcRows : (max_q <= 1 ? 1 : 4);
  const int groups = num_heads / hpc;
  const int smem = (tc ? kTcHeaderBytes : kHeaderBytes) + stages * stage_bytes;
  int ctas_per_sm = kSmemPerSM / (smem + 1024);
  const int thread_cap = 2048 / ((hpc + 1) * 32);
  ctas_per_sm = ctas_per_sm < 1 ? 1 : (ctas_per_sm > thread_cap ? thread_cap : ctas_per_sm);

  // split-K. A work item is (request, head group, query chunk, split); an item holds at most
  // kMaxBlocksPerSplit blocks (the shared-memory table slice). Rule fitted to sweeps on B200
  // measured as device time from CUDA-graph replays with L2 flushed (bf16, 16 heads x 64, 8-1024
  // requests x 1-4 rows, 128-4096 tokens, near-uniform and skewed lengths; 120 shapes): 1.016 x
  // the best split per shape on average, where the former rule was 1.11 x. (A 640-token cap
  // scored 1.018 x but left 592-token encoder contexts unsplit, 6-10 % slower at 128 requests.)
  //   * contexts of at most kNoSplitTokens, or three waves of unsplit items: no split;
  //   * fewer items: fill about 0.9 of a wave, with splits of at least kMinSplitTokens;
  //   * near-uniform long contexts: splits of at most kLongSplitTokens, so that many short items
  //     balance the SMs (the longest requests set the tail otherwise); skewed lengths: pieces
  //     of the total work over 1.5 waves (at least kSkewSplitTokens), whatever the fill;
  //   * then, for near-uniform lengths, no split count whose items land between one and two
  //     waves: the second wave's few CTAs cannot pull the bandwidth (e.g. 128 items x 4 splits,
  //     1.15 waves: 13 % slower than 3 splits, 0.86 waves) - back off to the most splits under
  //     one wave. Skewed items are no clean partial wave; there backing off cost up to 13 %.
  int64_t base_items = 0, sum_blocks = 0, busy_reqs = 0;
  for (int r = 0; r < num_reqs; ++r) {
    const int64_t ql = query_start_loc_host ? (int64_t)query_start_loc_host[r + 1] - query_start_loc_host[r] : 1;
    const int64_t qc = ceil_div(ql, (int64_t)qpc);
    const int64_t nb = ceil_div((int64_t)seq_lens_host[r], (int64_t)block_size);
    base_items += groups * qc;
    if (qc > 0 && nb > 0) {
      sum_blocks += nb;
      ++busy_reqs;
    }
  }
  const int64_t slots = (int64_t)kNumSMs * ctas_per_sm;
  const int64_t max_blocks = ceil_div(max_seq, (int64_t)block_size);
  const bool skewed = busy_reqs > 0 && 2 * max_blocks * busy_reqs > 3 * sum_blocks;  // max > 1.5 x mean
  // items of a split into pieces of `bps` blocks
  auto split_items_of = [&](int64_t bps) {
    int64_t items = 0;
    for (int r = 0; r < num_reqs; ++r) {
      const int64_t ql = query_start_loc_host ? (int64_t)query_start_loc_host[r + 1] - query_start_loc_host[r] : 1;
      items += ceil_div(ceil_div((int64_t)seq_lens_host[r], (int64_t)block_size), bps) * groups *
               ceil_div(ql, (int64_t)qpc);
    }
    return items;
  };
  const int64_t forced = ceil_div(max_blocks, (int64_t)kMaxBlocksPerSplit);  // the table slice's minimum
  int64_t want = 1;
  const int64_t max_tokens = max_blocks * block_size;
  if (max_tokens > kNoSplitTokens && base_items > 0 && base_items < 3 * slots) {
    int64_t fill = (9 * slots) / (10 * base_items);
    fill = fill < 1 ? 1 : fill;
    int64_t by_len = max_tokens / kMinSplitTokens;
    by_len = by_len < 1 ? 1 : by_len;
    want = fill < by_len ? fill : by_len;
    int64_t piece_tokens = kLongSplitTokens;
    if (skewed) {  // the work in tokens of all items, over 1.5 waves
      int64_t work = 0;
      for (int r = 0; r < num_reqs; ++r) {
        const int64_t ql = query_start_loc_host ? (int64_t)query_start_loc_host[r + 1] - query_start_loc_host[r] : 1;
        work += ceil_div((int64_t)seq_lens_host[r], (int64_t)block_size) * block_size * groups *
                ceil_div(ql, (int64_t)qpc);
      }
      piece_tokens = ceil_div(2 * work, 3 * slots);
      piece_tokens = piece_tokens < kSkewSplitTokens ? kSkewSplitTokens : piece_tokens;
    }
    const int64_t longest = ceil_div(max_tokens, piece_tokens);
    want = want > longest ? want : longest;
  }
  want = want < forced ? forced : want;
  int64_t bps = ceil_div(max_blocks, want);
  bps = bps < 1 ? 1 : (bps > kMaxBlocksPerSplit ? kMaxBlocksPerSplit : bps);
  while (!skewed && want > forced && want > 1) {  // skewed items are no clean partial wave
    const int64_t items = split_items_of(bps);
    if (items <= slots || items >= 2 * slots) break;
    --want;
    bps = ceil_div(max_blocks, want);
    bps = bps > kMaxBlocksPerSplit ? kMaxBlocksPerSplit : bps;
  }
  int64_t splits = ceil_div(max_blocks, bps);
  if (splits > 65535) {
    bps = ceil_div(max_blocks, (int64_t)65535);
    if (bps > kMaxBlocksPerSplit)
      return plan_fail(plan, fail(VFL_ERR_UNSUPPORTED, "sequence of %lld tokens is too long", (long long)max_seq));
    splits = ceil_div(max_blocks, bps);
  }
  // a full wave of short items: two stages per CTA (measured 3-11 % faster than four stages for
  // items of up to 256 tokens; mixed, within 10 % either way, at 577-592 tokens). The CTAs per
  // SM stay at three either way: the kernel's registers, not its shared memory, set them.
  if (base_items >= slots && bps * block_size <= kShortItemTokens && stages > 2) stages = 2;
  splits = splits < 1 ? 1 : splits;
  const int64_t q_chunks = ceil_div(max_q < 1 ? 1 : max_q, (int64_t)qpc);
  if (q_chunks > 65535 || (int64_t)num_reqs * groups > INT32_MAX)
    return plan_fail(plan, fail(VFL_ERR_UNSUPPORTED, "launch grid too large"));

  // Merge of split partials: a separate combine launch. The kernel can also merge in the
  // launch (the last split CTA of each item, behind an arrival counter; plan merge_in_kernel =
  // 1), but measured as device time that was slower in 1214 of 1220 swept cases (4-7 us per
  // call: the counters' memset and the merge on the tail's critical path).
  const int merge_in_kernel = 0;

  plan->magic = VFL_PLAN_MAGIC;
  plan->num_reqs = num_reqs;
  plan->num_heads = num_heads;
  plan->head_dim = head_dim;
  plan->block_size = block_size;
  plan->dtype = dtype;
  plan->causal = causal ? 1 : 0;
  plan->total_q = static_cast<int32_t>(total_q);
  plan->max_q_len = static_cast<int32_t>(max_q);
  plan->max_seq_len = static_cast<int32_t>(max_seq);
  plan->heads_per_cta = hpc;
  plan->queries_per_cta = qpc;
  plan->blocks_per_split = static_cast<int32_t>(bps);
  plan->num_splits = static_cast<int32_t>(splits);
  plan->stages = stages;
  plan->merge_in_kernel = merge_in_kernel;
  plan->row_tables = 0;
  set_schedule(plan, VFL_SCHEDULE_ITEMS, 0);  // sets workspace_bytes
  int64_t work = 0;  // 16-token tiles of all (request, head group) items
  for (int r = 0; r < num_reqs; ++r) {
    const int64_t ql = query_start_loc_host ? (int64_t)query_start_loc_host[r + 1] - query_start_loc_host[r] : 1;
    if (ql > 0) work += ceil_div((int64_t)seq_lens_host[r], (int64_t)16) * groups;
  }
  if (balanced_pays_off(plan, work, base_items, split_items_of(bps), splits, skewed)) {
    const int item_stages = plan->stages;
    plan->stages = 2;  // measured: two stages beat four in the balanced wave at every winning shape
    if (set_schedule(plan, VFL_SCHEDULE_BALANCED, 0) != VFL_OK) {
      plan->stages = item_stages;
      set_schedule(plan, VFL_SCHEDULE_ITEMS, 0);
    }
  }
  return VFL_OK;
}

int vfl_plan_attention_row_tables(int num_reqs, int num_heads, int num_kv_heads, int head_dim, int block_size,
                                  int dtype, const int32_t* seq_lens_host, const int32_t* query_start_loc_host,
                                  vfl_attention_plan* plan) {
  if (!use_tensor_cores(dtype, head_dim))
    return plan_fail(plan, fail(VFL_ERR_UNSUPPORTED, "row tables: built for bfloat16 with head_dim 64 only"));
  if (query_start_loc_host == nullptr && num_reqs > 0)
    return plan_fail(plan, fail(VFL_ERR_INVALID_ARGUMENT, "row tables: query_start_loc_host is NULL"));
  const int st = vfl_plan_attention(num_reqs, num_heads, num_kv_heads, head_dim, block_size, dtype, 0, seq_lens_host,
                                    query_start_loc_host, plan);
  if (st) return st;
  plan->row_tables = 1;
  return set_schedule(plan, VFL_SCHEDULE_ITEMS, 0);
}

int vfl_plan_attention_schedule(vfl_attention_plan* plan, int schedule, int min_tiles) {
  if (plan == nullptr || plan->magic != VFL_PLAN_MAGIC)
    return fail(VFL_ERR_INVALID_ARGUMENT, "plan_attention_schedule: plan missing or not built by vfl_plan_attention");
  const int st = check_attention_plan(plan);
  if (st) return st;
  return set_schedule(plan, schedule, min_tiles);
}

}  // extern "C"

namespace {

// The tokens a fused call appends: query row t's key / value rows and its slot.
struct AppendSource {
  const void* key;
  int64_t key_stride;
  const void* value;
  int64_t value_stride;
  const int64_t* slots;
};

int attention_run(const vfl_attention_plan* plan, const void* query, int64_t query_token_stride, const void* k_cache,
                  const void* v_cache, int64_t num_blocks, void* output, int64_t output_token_stride,
                  const int32_t* query_start_loc, const int32_t* seq_lens, const int32_t* block_table,
                  int64_t table_stride, int32_t table_cols, float scale, void* workspace, size_t workspace_bytes,
                  void* stream, const AppendSource* append) {
  if (plan == nullptr || plan->magic != VFL_PLAN_MAGIC)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: plan missing or not built by vfl_plan_attention");
  int st0 = check_attention_plan(plan);
  if (st0) return st0;
  const int H = plan->num_heads, D = plan->head_dim;
  if (plan->num_reqs == 0 || plan->total_q == 0) return VFL_OK;
  const int es = static_cast<int>(dtype_size(plan->dtype));
  if (!query || !k_cache || !v_cache || !output || !query_start_loc || !seq_lens || !block_table)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: NULL pointer");
  if (!aligned16(query) || !aligned16(output) || !aligned16(k_cache) || !aligned16(v_cache) ||
      (query_token_stride * es) % 16 != 0 || (output_token_stride * es) % 16 != 0)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: query/output/caches and token strides must be 16-byte aligned");
  if (query_token_stride < (int64_t)H * D || output_token_stride < (int64_t)H * D)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: token stride smaller than a token");
  if (num_blocks <= 0 || table_cols < 0 || table_stride < table_cols)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: bad pool or table sizes");
  if (plan->workspace_bytes > 0 &&
      (workspace == nullptr || workspace_bytes < static_cast<size_t>(plan->workspace_bytes) ||
       (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0))
    return fail(VFL_ERR_WORKSPACE, "attention: plan needs %lld workspace bytes (256-byte aligned), got %zu",
                (long long)plan->workspace_bytes, workspace_bytes);
  if ((int64_t)plan->max_seq_len > (int64_t)table_cols * plan->block_size)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention: seq_len %d exceeds the block table (%d blocks of %d)",
                plan->max_seq_len, table_cols, plan->block_size);

  AttnParams p{};
  p.q = query;
  p.q_stride = query_token_stride;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.num_blocks = num_blocks;
  p.out = output;
  p.out_stride = output_token_stride;
  p.qsl = query_start_loc;
  p.seq_lens = seq_lens;
  p.table = block_table;
  p.table_stride = table_stride;
  p.table_cols = table_cols;
  p.num_reqs = plan->num_reqs;
  p.total_q = plan->total_q;
  p.num_heads = H;
  p.block_size = plan->block_size;
  p.causal = plan->causal;
  p.heads_per_cta = plan->heads_per_cta;
  p.blocks_per_split = plan->blocks_per_split;
  p.num_splits = plan->num_splits;
  p.stages = plan->stages;
  p.max_seq_len = plan->max_seq_len;
  p.row_tables = plan->row_tables;
  p.schedule = plan->schedule;
  p.min_tiles = plan->min_tiles;
  p.balanced_ctas = plan->balanced_ctas;
  p.max_q_len = plan->max_q_len;
  p.scale_log2 = scale * 1.4426950408889634f;
  if (append != nullptr) {
    p.new_k = append->key;
    p.new_k_stride = append->key_stride;
    p.new_v = append->value;
    p.new_v_stride = append->value_stride;
    p.slots = append->slots;
  }
  int st = device_error_word(&p.err);
  if (st) return st;
  const int hpc = plan->heads_per_cta;
  const int qpc = plan->queries_per_cta;
  const int q_chunks = static_cast<int>(ceil_div(plan->max_q_len < 1 ? 1 : plan->max_q_len, qpc));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool balanced = plan->schedule == VFL_SCHEDULE_BALANCED;
  if (balanced) {
    const BalancedWorkspace w(plan->balanced_ctas, hpc, plan->num_reqs, H);
    char* base = static_cast<char*>(workspace);
    p.ws_acc = reinterpret_cast<float*>(base);
    p.ws_ml = reinterpret_cast<float*>(base + w.acc_bytes);
    p.ws_desc = reinterpret_cast<int4*>(base + w.acc_bytes + w.ml_bytes);
  } else if (plan->num_splits > 1) {
    const int64_t items = (int64_t)plan->total_q * H * plan->num_splits;
    const int64_t acc_bytes = ceil_div(items * D * 4, (int64_t)256) * 256;
    const int64_t ml_bytes = ceil_div(items * 2 * 4, (int64_t)256) * 256;
    char* base = static_cast<char*>(workspace);
    p.ws_acc = reinterpret_cast<float*>(base);
    p.ws_ml = reinterpret_cast<float*>(base + acc_bytes);
    if (plan->merge_in_kernel) {
      p.ws_arrivals = reinterpret_cast<int*>(base + acc_bytes + ml_bytes);
      const size_t counter_bytes = (size_t)plan->num_reqs * (H / hpc) * q_chunks * 4;
      st = cuda_status(cudaMemsetAsync(p.ws_arrivals, 0, counter_bytes, s), "cudaMemsetAsync(arrival counters)");
      if (st) return st;
    }
  }
  const dim3 grid = balanced ? dim3(plan->balanced_ctas) : dim3(plan->num_reqs * (H / hpc), plan->num_splits, q_chunks);
  const int threads = (hpc + 1) * 32;  // hpc consumer warps + one producer warp
  const bool tc = plan->queries_per_cta == kTcRows;
  const int smem = (tc ? kTcHeaderBytes : kHeaderBytes) + plan->stages * 2 * hpc * 16 * D * es +
                   (balanced ? balanced_sched_bytes(plan->num_reqs) : 0);
  if (tc) {
    const uint64_t rows = (uint64_t)num_blocks * H * plan->block_size;
    const uint32_t box_rows = plan->block_size == 16 ? 16u * hpc : 16u;
    CUtensorMap kmap, vmap;
    st = pool_tensor_map(k_cache, rows, box_rows, &kmap);
    if (st) return st;
    st = pool_tensor_map(v_cache, rows, box_rows, &vmap);
    if (st) return st;
    return launch_paged_attention_tc(p, kmap, vmap, grid, threads, smem, s);
  }
  if (plan->dtype == VFL_DTYPE_F32) return launch_paged_attention_f32(p, D, qpc, grid, threads, smem, s);
  return launch_paged_attention_bf16(p, D, qpc, grid, threads, smem, s);
}

}  // namespace

extern "C" {

int vfl_attention_with_kv_cache(const vfl_attention_plan* plan, const void* query,
                                int64_t query_token_stride, const void* k_cache,
                                const void* v_cache, int64_t num_blocks, void* output,
                                int64_t output_token_stride, const int32_t* query_start_loc,
                                const int32_t* seq_lens, const int32_t* block_table,
                                int64_t table_stride, int32_t table_cols, float scale,
                                void* workspace, size_t workspace_bytes, void* stream) {
  return attention_run(plan, query, query_token_stride, k_cache, v_cache, num_blocks, output, output_token_stride,
                       query_start_loc, seq_lens, block_table, table_stride, table_cols, scale, workspace,
                       workspace_bytes, stream, nullptr);
}

int vfl_attention_append_supported(const vfl_attention_plan* plan) {
  // Causal rows read the new tokens of earlier rows: all of a request's rows must be in one CTA
  // (one query chunk), or another CTA's stores would race this one's reads. Rows with their own
  // tables (beam groups) and single rows read only their own new token. The CUDA-core kernel
  // (float32, other head dims) appends for one row per request, the decode step's shape.
  if (plan == nullptr || plan->magic != VFL_PLAN_MAGIC) return 0;
  if (plan->queries_per_cta == kTcRows)
    return (plan->causal ? plan->max_q_len <= kTcRows : (plan->row_tables || plan->max_q_len <= 1)) ? 1 : 0;
  return plan->queries_per_cta == 1 && plan->max_q_len <= 1 ? 1 : 0;
}

int vfl_attention_with_kv_cache_append(const vfl_attention_plan* plan, const void* query,
                                       int64_t query_token_stride, const void* key, int64_t key_token_stride,
                                       const void* value, int64_t value_token_stride,
                                       const int64_t* slot_mapping, const void* k_cache, const void* v_cache,
                                       int64_t num_blocks, void* output, int64_t output_token_stride,
                                       const int32_t* query_start_loc, const int32_t* seq_lens,
                                       const int32_t* block_table, int64_t table_stride, int32_t table_cols,
                                       float scale, void* workspace, size_t workspace_bytes, void* stream) {
  if (plan == nullptr || plan->magic != VFL_PLAN_MAGIC)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention_append: plan missing or not built by vfl_plan_attention");
  if (!vfl_attention_append_supported(plan))
    return fail(VFL_ERR_UNSUPPORTED,
                "attention_append: built for one new token per query row: one row per request, or with the "
                "tensor-core kernel (bf16, head_dim 64) at most 8 causal rows per request or row tables");
  if (plan->num_reqs == 0 || plan->total_q == 0) return attention_run(plan, query, query_token_stride, k_cache,
      v_cache, num_blocks, output, output_token_stride, query_start_loc, seq_lens, block_table, table_stride,
      table_cols, scale, workspace, workspace_bytes, stream, nullptr);
  const int64_t row = (int64_t)plan->num_heads * plan->head_dim;
  if (!key || !value || !slot_mapping)
    return fail(VFL_ERR_INVALID_ARGUMENT, "attention_append: NULL key, value or slot_mapping");
  const int64_t es = (int64_t)dtype_size(plan->dtype);
  if (!aligned16(key) || !aligned16(value) || (key_token_stride * es) % 16 != 0 ||
      (value_token_stride * es) % 16 != 0 || key_token_stride < row || value_token_stride < row)
    return fail(VFL_ERR_INVALID_ARGUMENT,
                "attention_append: key/value must be 16-byte aligned with token strides of at least heads x head_dim");
  const AppendSource src{key, key_token_stride, value, value_token_stride, slot_mapping};
  return attention_run(plan, query, query_token_stride, k_cache, v_cache, num_blocks, output, output_token_stride,
                       query_start_loc, seq_lens, block_table, table_stride, table_cols, scale, workspace,
                       workspace_bytes, stream, &src);
}

}  // extern "C"
