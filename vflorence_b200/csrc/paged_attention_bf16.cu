// bfloat16 instantiations of the paged attention kernels (split from f32 to compile in parallel),
// including the tensor-core variant for head_dim 64 and its balanced schedule.
#include "paged_attention_balanced.cuh"

namespace vfl {
int launch_paged_attention_bf16(const AttnParams& p, int head_dim, int qpc, dim3 grid, int threads,
                                int smem_bytes, cudaStream_t stream) {
  return launch_dtype<__nv_bfloat16>(p, head_dim, qpc, grid, threads, smem_bytes, stream);
}

int launch_paged_attention_tc(const AttnParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap, dim3 grid,
                              int threads, int smem_bytes, cudaStream_t stream) {
  static int smem_done[kMaxDevices];
  // plans ask for at most kMaxStageBytes of ring unless they set more stages (checked on the host)
  const int want = smem_bytes > kTcHeaderBytes + kMaxStageBytes ? smem_bytes : kTcHeaderBytes + kMaxStageBytes;
  if (p.schedule == VFL_SCHEDULE_BALANCED) {
    static int smem_done_balanced[kMaxDevices];
    const int want_b = kTcHeaderBytes + kMaxStageBytes + balanced_sched_bytes(kBalancedMaxReqs);
    int st = ensure_smem_attribute(reinterpret_cast<const void*>(paged_attention_tc_balanced_kernel),
                                   smem_bytes > want_b ? smem_bytes : want_b, smem_done_balanced);
    if (st) return st;
    paged_attention_tc_balanced_kernel<<<grid, threads, smem_bytes, stream>>>(p, kmap, vmap);
    st = cuda_status(cudaGetLastError(), "paged_attention (balanced) launch");
    if (st) return st;
    // the merge of cut items as a programmatic dependent launch: its CTAs start while the
    // attention grid drains and wait for it (griddepcontrol.wait) before reading the pieces
    return launch_dependent(paged_attention_tc_balanced_combine_kernel,
                            dim3(static_cast<unsigned>(p.num_reqs * (p.num_heads / p.heads_per_cta)),
                                 static_cast<unsigned>(p.max_q_len < 1 ? 1 : p.max_q_len)),
                            dim3(static_cast<unsigned>(32 * p.heads_per_cta)), stream,
                            "paged_attention (balanced) merge launch", p);
  }
  int st = ensure_smem_attribute(reinterpret_cast<const void*>(paged_attention_tc_kernel), want, smem_done);
  if (st) return st;
  paged_attention_tc_kernel<<<grid, threads, smem_bytes, stream>>>(p, kmap, vmap);
  st = cuda_status(cudaGetLastError(), "paged_attention (tensor cores) launch");
  if (st || p.num_splits <= 1 || p.ws_arrivals != nullptr) return st;
  const int64_t warps = (int64_t)p.total_q * p.num_heads;
  return launch_dependent(paged_attention_combine_kernel<__nv_bfloat16, 64>,
                          dim3(static_cast<unsigned>(ceil_div(warps, (int64_t)4))), dim3(128), stream,
                          "paged_attention combine launch", p);
}
}  // namespace vfl
