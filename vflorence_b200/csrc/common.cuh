// Shared helpers for the vflorence_b200 kernels (sm_100a): host-side status plumbing and the
// few PTX forms the kernels use (mbarrier, bulk global->shared copies, bounded waits).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>

#include "vflorence_b200.h"

namespace vfl {

// ------------------------------------------------------------------ host-side status plumbing

// Records a printf-style message as this thread's last error and returns `status`.
int fail(int status, const char* fmt, ...);
// Returns VFL_OK, or VFL_ERR_CUDA with the runtime's message when `e` is an error.
int cuda_status(cudaError_t e, const char* what);
// Device address of the current device's error word (set up once per device).
int device_error_word(unsigned int** out);
// A row-major bf16 matrix as a 2-D TMA tensor map (128-byte swizzle, zero fill outside).
int make_tensor_map_2d_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                            uint32_t box_outer, CUtensorMap* out);
// Re-checks every field of a caller-provided attention plan that the kernels rely on.
int check_attention_plan(const vfl_attention_plan* plan);
// Raises the dynamic shared-memory limit of `func` once per device.
int ensure_smem_attribute(const void* func, int bytes, int* done_flags /* [kMaxDevices] */);

constexpr int kMaxDevices = 64;
// B200: 148 SMs on two dies. The planner sizes grids for this count.
constexpr int kNumSMs = 148;

inline size_t dtype_size(int dtype) { return dtype == VFL_DTYPE_F32 ? 4u : 2u; }
inline bool dtype_ok(int dtype) { return dtype == VFL_DTYPE_F32 || dtype == VFL_DTYPE_BF16; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
template <typename A, typename B>
__host__ __device__ constexpr A ceil_div(A a, B b) {
  return (a + b - 1) / b;
}
__host__ __device__ constexpr int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Head dims the attention kernels are built for (the reference's list,
// vflorence/layers/attention.py:6).
inline bool head_dim_supported(int d) {
  switch (d) {
    case 32: case 48: case 64: case 80: case 96: case 112: case 128:
    case 160: case 192: case 224: case 256: case 512:
      return true;
    default:
      return false;
  }
}

// ------------------------------------------------------------------ device helpers

__device__ __forceinline__ void report(unsigned int* err, unsigned int bits) {
  if (err != nullptr) atomicOr(err, bits);
}

// Programmatic dependent launch. The grid launched next on the stream as this grid's
// programmatic dependent may start once every CTA here has called launch_dependents (or
// exited); griddepcontrol.wait in the dependent blocks until this grid has completed and its
// memory operations are visible. A grid launched without the attribute waits as usual, and
// griddepcontrol.wait then returns at once.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ unsigned int load_volatile(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async proxy (bulk copies complete on it).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}


__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Bulk (non-tensor) copy global -> shared, completion signalled on `bar` as transaction bytes.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// L2 policy for data read exactly once (K/V tiles): evict it first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// L2 policy for data other CTAs read soon after (blocks shared by the beams of a request).
__device__ __forceinline__ uint64_t l2_evict_normal_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// bulk_copy_g2s with an L2 cache-policy hint.
__device__ __forceinline__ void bulk_copy_g2s_hint(void* dst, const void* src, uint32_t bytes,
                                                   uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for phase `parity` of `bar` to complete; gives up after `limit_ns` of wall time
// (kWaitLimitNs unless a caller passes a shorter one) and returns false (the caller records
// VFL_DEVERR_TIMEOUT and unwinds without faulting).
constexpr uint64_t kWaitLimitNs = 2000000000ull;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = kWaitLimitNs) {
#pragma unroll 1
  for (int i = 0; i < 64; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// 16-byte read-only global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// d{0,1} += a{0,1} * b{0,1} as one packed two-lane fp32 FMA (sm_100 f32x2 arithmetic).
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 a, b, c;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%0, %1};\n\t"
      "fma.rn.f32x2 c, a, b, c;\n\tmov.b64 {%0, %1}, c;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// 2^x with the hardware approximation (one MUFU op; subnormal results flush to zero).
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------------------------ element conversion

template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static constexpr int kVec = 4;  // elements per 16-byte vector
};
template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;
};

// 16 bytes -> kVec floats.
__device__ __forceinline__ void unpack16(const uint4& v, float* f, float /*tag*/) {
  f[0] = __uint_as_float(v.x);
  f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z);
  f[3] = __uint_as_float(v.w);
}
__device__ __forceinline__ void unpack16(const uint4& v, float* f, __nv_bfloat16 /*tag*/) {
  f[0] = __uint_as_float(v.x << 16);
  f[1] = __uint_as_float(v.x & 0xffff0000u);
  f[2] = __uint_as_float(v.y << 16);
  f[3] = __uint_as_float(v.y & 0xffff0000u);
  f[4] = __uint_as_float(v.z << 16);
  f[5] = __uint_as_float(v.z & 0xffff0000u);
  f[6] = __uint_as_float(v.w << 16);
  f[7] = __uint_as_float(v.w & 0xffff0000u);
}

// kVec floats -> 16 bytes (bf16: round to nearest even).
__device__ __forceinline__ uint4 pack16(const float* f, float /*tag*/) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint4 pack16(const float* f, __nv_bfloat16 /*tag*/) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

}  // namespace vfl
