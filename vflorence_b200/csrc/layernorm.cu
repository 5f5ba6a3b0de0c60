// Residual add fused with LayerNorm: out[r] = LayerNorm(h[r] + x[r]) * weight + bias - the
// post-norm residual that closes every sub-layer of the BART decoder the paged ops serve
// (vflorence/models/bart.py:192-201: self_attn_layer_norm(h + attn), encoder_attn_layer_norm
// (h + cross), final_layer_norm(h + ffn)), and the embedding's layernorm_embedding(tok + pos)
// (bart.py:260-264). In the decode step these run on [rows <= 256, d_model] tensors, where the
// separate add and norm launches cost latency, not bandwidth.
//
// One warp per row; each lane keeps d / 32 elements in registers as 16-byte vectors (so d must
// be a multiple of 32 vectors: 256 for bf16, 128 for fp32). The sum is rounded to the tensor's
// dtype first, as the separate add does; mean and variance are two-pass fp32 over the
// registers (biased variance, as torch.nn.LayerNorm), then y = (s - mean) * rstd * w + b in
// fp32, rounded once.
#include "common.cuh"

namespace vfl {
namespace {

constexpr int kRowsPerBlock = 4;  // warps per block, one row each

template <typename T>
struct Vec;
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float (&f)[4]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    f[0] = v.x, f[1] = v.y, f[2] = v.z, f[3] = v.w;
  }
  __device__ static float round(float v) { return v; }
  __device__ static void store(float* p, const float (&f)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
};
template <>
struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float (&f)[8]) {
    unpack16(*reinterpret_cast<const uint4*>(p), f, __nv_bfloat16{});
  }
  __device__ static float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
  __device__ static void store(__nv_bfloat16* p, const float (&f)[8]) {
    *reinterpret_cast<uint4*>(p) = pack16(f, __nv_bfloat16{});
  }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// V = 16-byte vectors per lane; d = 32 * V * Vec<T>::N.
template <typename T, int V>
__global__ void __launch_bounds__(kRowsPerBlock * 32) add_layernorm_kernel(
    const T* h, int64_t h_stride, const T* x, int64_t x_stride, const T* __restrict__ w,
    const T* __restrict__ b, T* out, int64_t out_stride, int rows, float eps) {
  // out may alias h or x: each lane reads all of its elements before it writes any
  constexpr int E = Vec<T>::N;
  constexpr int d = 32 * V * E;
  const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float s[V][E];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = (i * 32 + lane) * E;
    float hv[E], xv[E];
    Vec<T>::load(h + row * h_stride + c, hv);
    Vec<T>::load(x + row * x_stride + c, xv);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      s[i][e] = Vec<T>::round(hv[e] + xv[e]);
      sum += s[i][e];
    }
  }
  const float mean = warp_sum(sum) * (1.f / d);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float c = s[i][e] - mean;
      sq = fmaf(c, c, sq);
    }
  const float rstd = rsqrtf(warp_sum(sq) * (1.f / d) + eps);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = (i * 32 + lane) * E;
    float wv[E], bv[E], y[E];
    Vec<T>::load(w + c, wv);
    if (b != nullptr) {
      Vec<T>::load(b + c, bv);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) bv[e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < E; ++e) y[e] = fmaf((s[i][e] - mean) * rstd, wv[e], bv[e]);
    Vec<T>::store(out + row * out_stride + c, y);
  }
}

template <typename T, int V>
int launch_add_layernorm(const void* h, int64_t hs, const void* x, int64_t xs, const void* w, const void* b,
                         void* out, int64_t os, int rows, float eps, cudaStream_t stream) {
  const int grid = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  add_layernorm_kernel<T, V><<<grid, kRowsPerBlock * 32, 0, stream>>>(
      static_cast<const T*>(h), hs, static_cast<const T*>(x), xs, static_cast<const T*>(w),
      static_cast<const T*>(b), static_cast<T*>(out), os, rows, eps);
  return cuda_status(cudaGetLastError(), "add_layernorm launch");
}

template <typename T>
int dispatch_add_layernorm(int v, const void* h, int64_t hs, const void* x, int64_t xs, const void* w,
                           const void* b, void* out, int64_t os, int rows, float eps, cudaStream_t s) {
  switch (v) {
    case 1: return launch_add_layernorm<T, 1>(h, hs, x, xs, w, b, out, os, rows, eps, s);
    case 2: return launch_add_layernorm<T, 2>(h, hs, x, xs, w, b, out, os, rows, eps, s);
    case 3: return launch_add_layernorm<T, 3>(h, hs, x, xs, w, b, out, os, rows, eps, s);
    case 4: return launch_add_layernorm<T, 4>(h, hs, x, xs, w, b, out, os, rows, eps, s);
    case 5: return launch_add_layernorm<T, 5>(h, hs, x, xs, w, b, out, os, rows, eps, s);
    case 6: return launch_add_layernorm<T, 6>(h, hs, x, xs, w, b, out, os, rows, eps, s);
    case 7: return launch_add_layernorm<T, 7>(h, hs, x, xs, w, b, out, os, rows, eps, s);
    case 8: return launch_add_layernorm<T, 8>(h, hs, x, xs, w, b, out, os, rows, eps, s);
    default: return VFL_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace vfl

using namespace vfl;

extern "C" int vfl_add_layernorm_supported(int dtype, int hidden_dim) {
  if (!dtype_ok(dtype) || hidden_dim <= 0) return 0;
  const int per_warp = 32 * (16 / (int)dtype_size(dtype));  // elements in one vector per lane
  return hidden_dim % per_warp == 0 && hidden_dim / per_warp <= 8 ? 1 : 0;
}

extern "C" int vfl_add_layernorm(const void* h, int64_t h_stride, const void* x, int64_t x_stride,
                                 const void* weight, const void* bias, void* out, int64_t out_stride,
                                 int32_t rows, int32_t hidden_dim, float eps, int32_t dtype, void* stream) {
  if (!dtype_ok(dtype)) return fail(VFL_ERR_INVALID_ARGUMENT, "add_layernorm: dtype %d", dtype);
  if (rows < 0 || hidden_dim <= 0 || !(eps >= 0.f))
    return fail(VFL_ERR_INVALID_ARGUMENT, "add_layernorm: rows %d, hidden_dim %d, eps %g", rows, hidden_dim,
                (double)eps);
  if (!vfl_add_layernorm_supported(dtype, hidden_dim))
    return fail(VFL_ERR_UNSUPPORTED, "add_layernorm: hidden_dim %d is not a multiple of 32 16-byte vectors (at most 8 "
                "per lane)", hidden_dim);
  if (rows == 0) return VFL_OK;
  if (!h || !x || !weight || !out) return fail(VFL_ERR_INVALID_ARGUMENT, "add_layernorm: NULL pointer");
  const int64_t es = (int64_t)dtype_size(dtype);
  if (!aligned16(h) || !aligned16(x) || !aligned16(weight) || !aligned16(out) || (bias && !aligned16(bias)) ||
      (h_stride * es) % 16 || (x_stride * es) % 16 || (out_stride * es) % 16 || h_stride < hidden_dim ||
      x_stride < hidden_dim || out_stride < hidden_dim)
    return fail(VFL_ERR_INVALID_ARGUMENT,
                "add_layernorm: pointers and row strides must be 16-byte aligned, strides >= hidden_dim");
  const int v = hidden_dim / (32 * (int)(16 / es));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == VFL_DTYPE_F32)
    return dispatch_add_layernorm<float>(v, h, h_stride, x, x_stride, weight, bias, out, out_stride, rows, eps, s);
  return dispatch_add_layernorm<__nv_bfloat16>(v, h, h_stride, x, x_stride, weight, bias, out, out_stride, rows, eps,
                                               s);
}
