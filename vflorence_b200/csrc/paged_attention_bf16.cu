// bfloat16 instantiations of the paged attention kernels (split from f32 to compile in parallel).
#include "paged_attention_kernels.cuh"

namespace vfl {
int launch_paged_attention_bf16(const AttnParams& p, int head_dim, int qpc, dim3 grid, int threads,
                                int smem_bytes, cudaStream_t stream) {
  return launch_dtype<__nv_bfloat16>(p, head_dim, qpc, grid, threads, smem_bytes, stream);
}
}  // namespace vfl
