"""vflorence_b200: the paged-KV attention path of the vflorence engine, on B200 (sm_100a).

Modules
    paged_ops      the vllm_cpu_attn functions (get_isa, get_scheduler_metadata,
                   reshape_and_cache, attention_with_kv_cache) + copy_blocks, prepare_decode,
                   paged_slots - thin Python over the C ABI in include/vflorence_b200.h
    attention      the vflorence::self_attention / vflorence::cross_attention custom ops and
                   stage_cross (imported on demand: importing it registers the ops)
    context        the per-step Context the ops read
    block_manager  the host-side block allocator whose outputs the kernels consume
    kv_cache       device-resident pools, encoder pages, copy-on-write and per-step metadata
    build          nvcc recipe for the in-tree library
"""

from . import paged_ops
from .block_manager import BlockManager

__all__ = ["paged_ops", "BlockManager"]
__version__ = "0.1.0"
