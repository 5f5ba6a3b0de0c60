// vfl_attention_with_kv_cache_no_alloc: paged attention whose split-K scratch lives in a fixed
// array compiled into this library, for callers that cannot allocate device memory.
//
// Who needs it: a C or C++ host that binds the ABI directly (a serving loop, an FFI host)
// usually has no device allocator of its own - every scratch buffer would be a cudaMalloc,
// which synchronises the device and stalls the decode loop - and some processes hand all
// device memory to a framework's pool up front, so a side allocation can fail outright. This
// entry point takes no workspace argument: the scratch is the array below.
//
// Limits and sharing:
//   * The array holds VFL_STATIC_WORKSPACE_BYTES (64 MiB). Every device that loads this code
//     keeps that much memory until the process exits. A plan whose workspace_bytes is larger
//     is rejected with VFL_ERR_WORKSPACE before anything is launched.
//   * Every call on a device uses the same array, and it keeps whatever the last call left in
//     it. The plans vfl_plan_attention builds merge the split-K partials in a separate combine
//     launch and keep no state in the array between calls: every partial the combine reads was
//     written earlier in the same call. Only a caller-built plan with merge_in_kernel = 1 puts
//     per-request arrival counters in the array (they pick the CTA that merges); those must
//     start at zero, and such a call clears them on its stream before its kernel runs. Calls
//     whose kernels can overlap on one device (for example on two streams without an ordering
//     between them) race on the array and give wrong results; order them on one stream or with
//     events.
//   * The first call on each device looks up the array's device address (cudaGetSymbolAddress,
//     with that device current) and caches it for the life of the process; make that first
//     call before any stream capture. The cache does not survive cudaDeviceReset (the module
//     reloads and the array may move): do not use this entry point after resetting a device.
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace {

// The scratch. In host code this name is only a stand-in for the symbol, never a usable
// address: the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_static_workspace[VFL_STATIC_WORKSPACE_BYTES];

std::atomic<void*> g_static_workspace_addr[vfl::kMaxDevices];
std::mutex g_static_workspace_mutex;

// Device address of the current device's array, looked up once per device.
int static_workspace_address(void** out) {
  int dev = 0;
  int st = vfl::cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (st) return st;
  if (dev < 0 || dev >= vfl::kMaxDevices)
    return vfl::fail(VFL_ERR_CUDA, "device ordinal %d out of range", dev);
  void* p = g_static_workspace_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_static_workspace_mutex);
    p = g_static_workspace_addr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      void* addr = nullptr;
      st = vfl::cuda_status(cudaGetSymbolAddress(&addr, g_static_workspace),
                            "cudaGetSymbolAddress(static attention workspace)");
      if (st) return st;
      p = addr;
      g_static_workspace_addr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return VFL_OK;
}

}  // namespace

extern "C" int vfl_attention_with_kv_cache_no_alloc(
    const vfl_attention_plan* plan, const void* query, int64_t query_token_stride,
    const void* k_cache, const void* v_cache, int64_t num_blocks, void* output,
    int64_t output_token_stride, const int32_t* query_start_loc, const int32_t* seq_lens,
    const int32_t* block_table, int64_t table_stride, int32_t table_cols, float scale,
    void* stream) {
  if (plan == nullptr || plan->magic != VFL_PLAN_MAGIC)
    return vfl::fail(VFL_ERR_INVALID_ARGUMENT,
                     "attention (no alloc): plan missing or not built by vfl_plan_attention");
  int st0 = vfl::check_attention_plan(plan);
  if (st0) return st0;
  if (plan->workspace_bytes > (int64_t)VFL_STATIC_WORKSPACE_BYTES)
    return vfl::fail(VFL_ERR_WORKSPACE,
                     "attention (no alloc): this plan needs %lld bytes of split-K scratch but the "
                     "built-in scratch holds %lld; split the batch or call "
                     "vfl_attention_with_kv_cache with a workspace",
                     (long long)plan->workspace_bytes, (long long)VFL_STATIC_WORKSPACE_BYTES);
  void* ws = nullptr;
  int st = static_workspace_address(&ws);
  if (st) return st;
  return vfl_attention_with_kv_cache(plan, query, query_token_stride, k_cache, v_cache, num_blocks,
                                     output, output_token_stride, query_start_loc, seq_lens,
                                     block_table, table_stride, table_cols, scale, ws,
                                     VFL_STATIC_WORKSPACE_BYTES, stream);
}
