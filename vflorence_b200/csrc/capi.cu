// Library-level C ABI: status strings, the thread-local last-error message, the per-device
// error word that kernels report into, and get_isa.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {

thread_local char g_last_error[512] = "";

// One word per device (a __device__ variable has one instance per device context). Kernels
// atomicOr VFL_DEVERR_* bits into it; vfl_read_device_errors reads and clears it.
__device__ unsigned int g_device_error_word = 0;

std::atomic<unsigned int*> g_error_word_addr[vfl::kMaxDevices];
std::mutex g_setup_mutex;

// The bounded-wait path of the pipelined kernels, on its own: warp 0 waits (bounded) on a
// shared-memory barrier that expects one arrival; warp 1 plays the producer and makes that
// arrival only when `arrive` is set. Without it the wait gives up after `limit_ns`, warp 0
// reports VFL_DEVERR_TIMEOUT and raises the CTA's abort flag, and both warps meet at the CTA
// barrier and exit - the unwinding the attention kernels use.
__global__ void __launch_bounds__(64) bounded_wait_check_kernel(int arrive, uint64_t limit_ns,
                                                                unsigned int* err) {
  __shared__ uint64_t full;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    vfl::mbar_init(&full, 1);
    abort_flag = 0;
    vfl::fence_barrier_init();
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 1) {
    if (arrive && lane == 0) vfl::mbar_arrive(&full);
  } else if (lane == 0 && !vfl::mbar_wait_bounded(&full, 0, limit_ns)) {
    vfl::report(err, VFL_DEVERR_TIMEOUT);
    abort_flag = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag == 0 && !arrive) vfl::report(err, VFL_DEVERR_QUERY);  // cannot happen
}

}  // namespace

namespace vfl {

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return VFL_OK;
  return fail(VFL_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int device_error_word(unsigned int** out) {
  int dev = 0;
  int st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (st) return st;
  if (dev < 0 || dev >= kMaxDevices) return fail(VFL_ERR_CUDA, "device ordinal %d out of range", dev);
  unsigned int* p = g_error_word_addr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    p = g_error_word_addr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      void* addr = nullptr;
      st = cuda_status(cudaGetSymbolAddress(&addr, g_device_error_word), "cudaGetSymbolAddress(error word)");
      if (st) return st;
      p = static_cast<unsigned int*>(addr);
      g_error_word_addr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return VFL_OK;
}

int ensure_smem_attribute(const void* func, int bytes, int* done_flags) {
  int dev = 0;
  int st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (st) return st;
  if (dev < 0 || dev >= kMaxDevices) return fail(VFL_ERR_CUDA, "device ordinal %d out of range", dev);
  if (__atomic_load_n(&done_flags[dev], __ATOMIC_ACQUIRE) >= bytes) return VFL_OK;
  st = cuda_status(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                   "cudaFuncSetAttribute(max dynamic shared memory)");
  if (st) return st;
  __atomic_store_n(&done_flags[dev], bytes, __ATOMIC_RELEASE);
  return VFL_OK;
}

}  // namespace vfl

extern "C" {

int vfl_abi_version(void) { return VFL_ABI_VERSION; }

const char* vfl_status_string(int status) {
  switch (status) {
    case VFL_OK: return "ok";
    case VFL_ERR_INVALID_ARGUMENT: return "invalid argument";
    case VFL_ERR_UNSUPPORTED: return "unsupported configuration";
    case VFL_ERR_WORKSPACE: return "workspace missing or too small";
    case VFL_ERR_CUDA: return "CUDA runtime error";
    case VFL_ERR_CAPACITY: return "capacity exhausted";
    default: return "unknown status";
  }
}

const char* vfl_last_error_message(void) { return g_last_error; }

int vfl_read_device_errors(unsigned int* bits, int clear, void* stream) {
  if (bits == nullptr) return vfl::fail(VFL_ERR_INVALID_ARGUMENT, "bits is NULL");
  unsigned int* word = nullptr;
  int st = vfl::device_error_word(&word);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int host = 0;
  st = vfl::cuda_status(cudaMemcpyAsync(&host, word, sizeof(host), cudaMemcpyDeviceToHost, s),
                        "cudaMemcpyAsync(error word)");
  if (st) return st;
  if (clear) {
    st = vfl::cuda_status(cudaMemsetAsync(word, 0, sizeof(unsigned int), s), "cudaMemsetAsync(error word)");
    if (st) return st;
  }
  st = vfl::cuda_status(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  if (st) return st;
  *bits = host;
  return VFL_OK;
}

int vfl_check_bounded_wait(int producer_arrives, int64_t limit_ns, void* stream) {
  if (limit_ns <= 0 || limit_ns > static_cast<int64_t>(vfl::kWaitLimitNs))
    return vfl::fail(VFL_ERR_INVALID_ARGUMENT, "limit_ns %lld: must be in (0, %llu]",
                     static_cast<long long>(limit_ns), static_cast<unsigned long long>(vfl::kWaitLimitNs));
  unsigned int* err = nullptr;
  int st = vfl::device_error_word(&err);
  if (st) return st;
  bounded_wait_check_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      producer_arrives != 0, static_cast<uint64_t>(limit_ns), err);
  return vfl::cuda_status(cudaGetLastError(), "bounded_wait_check_kernel launch");
}

int vfl_get_isa(int dtype, int block_size, int head_dim, char* buf, int buf_len) {
  if (!vfl::dtype_ok(dtype))
    return vfl::fail(VFL_ERR_UNSUPPORTED, "dtype %d: only float32 and bfloat16 are built", dtype);
  if (block_size < 16 || block_size % 16 != 0 || block_size > 1024)
    return vfl::fail(VFL_ERR_UNSUPPORTED, "block_size %d: must be a multiple of 16 in [16, 1024]",
                     block_size);
  if (!vfl::head_dim_supported(head_dim))
    return vfl::fail(VFL_ERR_UNSUPPORTED,
                     "head_dim %d: the sm100 kernels cover 32, 48, 64, 80, 96, 112, 128, 160, "
                     "192, 224, 256 and 512",
                     head_dim);
  if (buf == nullptr || buf_len < 6) return vfl::fail(VFL_ERR_INVALID_ARGUMENT, "buffer too small");
  std::memcpy(buf, "sm100", 6);
  return VFL_OK;
}

}  // extern "C"
