"""ctypes binding of ``libvflorence_b200.so`` (the C ABI declared in ``include/vflorence_b200.h``
and ``include/vflorence_b200_runtime.h``).

This is the whole Python<->native boundary: plain pointers, sizes and a stream handle go in, a
status code comes out. A missing or unloadable library raises at first use - there is no
fallback path.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libvflorence_b200.so")

VFL_OK = 0
VFL_ERR_INVALID_ARGUMENT = 1
VFL_ERR_UNSUPPORTED = 2
VFL_ERR_WORKSPACE = 3
VFL_ERR_CUDA = 4
VFL_ERR_CAPACITY = 5
ABI_VERSION = 4

DTYPE_F32 = 0
DTYPE_BF16 = 1

DEVERR_BLOCK_ID = 0x1
DEVERR_SLOT = 0x2
DEVERR_CONTEXT = 0x4
DEVERR_TIMEOUT = 0x8
DEVERR_QUERY = 0x10

PLAN_MAGIC = 0x31504C4656
MAX_COPY_LAYERS = 128
STATIC_WORKSPACE_BYTES = 64 * 1024 * 1024

# Every exported entry point of the C ABI, in header order.
EXPORTS = (
    "vfl_abi_version",
    "vfl_status_string",
    "vfl_last_error_message",
    "vfl_read_device_errors",
    "vfl_check_bounded_wait",
    "vfl_get_isa",
    "vfl_plan_attention",
    "vfl_plan_attention_row_tables",
    "vfl_plan_attention_schedule",
    "vfl_reshape_and_cache",
    "vfl_attention_with_kv_cache",
    "vfl_attention_with_kv_cache_append",
    "vfl_attention_append_supported",
    "vfl_attention_with_kv_cache_no_alloc",
    "vfl_copy_blocks",
    "vfl_prepare_decode",
    "vfl_kv_proj_paged",
    "vfl_add_layernorm",
    "vfl_add_layernorm_supported",
    "vfl_decode_linear",
    "vfl_decode_linear_supported",
    "vfl_paged_slots",
    "vfl_row_topk",
    "vfl_row_topk_workspace_size",
    "vfl_beam_merge",
    "vfl_fork_token_rows",
    # host decode runtime (vflorence_b200_runtime.h)
    "vfl_rt_create",
    "vfl_rt_destroy",
    "vfl_rt_reset",
    "vfl_rt_slot_acquire",
    "vfl_rt_slot_release",
    "vfl_rt_num_free_blocks",
    "vfl_rt_free_block_ids",
    "vfl_rt_ref_count",
    "vfl_rt_block_table",
    "vfl_rt_required_new_blocks",
    "vfl_rt_ensure_capacity",
    "vfl_rt_fork",
    "vfl_rt_deallocate",
    "vfl_rt_admit",
    "vfl_rt_num_running",
    "vfl_rt_prepare_step",
    "vfl_rt_pack_step",
    "vfl_rt_advance_greedy",
    "vfl_rt_advance_beam",
)


class AttentionPlan(ctypes.Structure):
    """Mirror of ``vfl_attention_plan``."""

    _fields_ = [
        ("magic", ctypes.c_int64),
        ("num_reqs", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("total_q", ctypes.c_int32),
        ("max_q_len", ctypes.c_int32),
        ("max_seq_len", ctypes.c_int32),
        ("heads_per_cta", ctypes.c_int32),
        ("queries_per_cta", ctypes.c_int32),
        ("blocks_per_split", ctypes.c_int32),
        ("num_splits", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("merge_in_kernel", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_int64),
        ("row_tables", ctypes.c_int32),
        ("schedule", ctypes.c_int32),
        ("min_tiles", ctypes.c_int32),
        ("balanced_ctas", ctypes.c_int32),
    ]


PLAN_BYTES = ctypes.sizeof(AttentionPlan)


class DecodeRules(ctypes.Structure):
    """Mirror of ``vfl_decode_rules``."""

    _fields_ = [
        ("num_beams", ctypes.c_int32),
        ("max_tokens", ctypes.c_int32),
        ("length_penalty", ctypes.c_double),
        ("early_stopping", ctypes.c_int32),
        ("num_eos", ctypes.c_int32),
        ("eos_ids", ctypes.c_void_p),
    ]


class StepResult(ctypes.Structure):
    """Mirror of ``vfl_step_result``."""

    _fields_ = [
        ("born_parent", ctypes.c_void_p),
        ("born_child", ctypes.c_void_p),
        ("born_pos", ctypes.c_void_p),
        ("born_token", ctypes.c_void_p),
        ("born_cap", ctypes.c_int32),
        ("num_born", ctypes.c_int32),
        ("done_request", ctypes.c_void_p),
        ("done_slot", ctypes.c_void_p),
        ("done_length", ctypes.c_void_p),
        ("done_cap", ctypes.c_int32),
        ("num_done", ctypes.c_int32),
    ]


class VflError(RuntimeError):
    """A failing C-ABI call; ``status`` is the vfl_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_lock = threading.Lock()
_lib = None


def _declare(L):
    vp, i32, i64, f32, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
    plan_p = ctypes.POINTER(AttentionPlan)
    sig = {
        "vfl_abi_version": (i32, []),
        "vfl_status_string": (ctypes.c_char_p, [i32]),
        "vfl_last_error_message": (ctypes.c_char_p, []),
        "vfl_read_device_errors": (i32, [ctypes.POINTER(ctypes.c_uint), i32, vp]),
        "vfl_check_bounded_wait": (i32, [i32, i64, vp]),
        "vfl_get_isa": (i32, [i32, i32, i32, ctypes.c_char_p, i32]),
        "vfl_plan_attention": (i32, [i32, i32, i32, i32, i32, i32, i32, vp, vp, plan_p]),
        "vfl_plan_attention_row_tables": (i32, [i32, i32, i32, i32, i32, i32, vp, vp, plan_p]),
        "vfl_plan_attention_schedule": (i32, [plan_p, i32, i32]),
        "vfl_reshape_and_cache": (i32, [vp, vp, vp, vp, vp, i64, i32, i32, i32, i64, i64, i64, i32, vp]),
        "vfl_attention_with_kv_cache": (i32, [vp, vp, i64, vp, vp, i64, vp, i64, vp, vp, vp, i64, i32,
                                              f32, vp, sz, vp]),
        "vfl_attention_with_kv_cache_append": (i32, [plan_p, vp, i64, vp, i64, vp, i64, vp, vp, vp, i64, vp, i64, vp,
                                                     vp, vp, i64, i32, f32, vp, sz, vp]),
        "vfl_attention_append_supported": (i32, [plan_p]),
        "vfl_attention_with_kv_cache_no_alloc": (i32, [plan_p, vp, i64, vp, vp, i64, vp, i64, vp, vp, vp,
                                                       i64, i32, f32, vp]),
        "vfl_copy_blocks": (i32, [vp, vp, i32, vp, i32, i64, i64, vp]),
        "vfl_prepare_decode": (i32, [vp, i64, i32, vp, i32, i32, vp, vp, vp, vp]),
        "vfl_paged_slots": (i32, [vp, i64, i32, i32, i32, i32, vp, vp]),
        "vfl_kv_proj_paged": (i32, [vp, i64, vp, vp, vp, vp, vp, i64, i32, i32, i32, i32, i64, vp]),
        "vfl_add_layernorm": (i32, [vp, i64, vp, i64, vp, vp, vp, i64, i32, i32, f32, i32, vp]),
        "vfl_add_layernorm_supported": (i32, [i32, i32]),
        "vfl_decode_linear": (i32, [vp, i64, vp, vp, vp, i64, i32, i32, i32, i32, i32, vp]),
        "vfl_decode_linear_supported": (i32, [i32, i32, i32, i32]),
        "vfl_row_topk": (i32, [vp, i32, i64, i64, i64, i32, vp, i32, vp, vp, vp, sz, vp]),
        "vfl_row_topk_workspace_size": (sz, [i64, i64, i32]),
        "vfl_beam_merge": (i32, [vp, vp, i64, i32, vp, vp, i32, i32, vp, vp]),
        "vfl_fork_token_rows": (i32, [vp, i64, i32, i32, vp, i32, vp]),
        "vfl_rt_create": (i32, [i32, i32, i32, i32, ctypes.POINTER(vp)]),
        "vfl_rt_destroy": (None, [vp]),
        "vfl_rt_reset": (i32, [vp]),
        "vfl_rt_slot_acquire": (i32, [vp, vp]),
        "vfl_rt_slot_release": (i32, [vp, i32]),
        "vfl_rt_num_free_blocks": (i32, [vp, vp]),
        "vfl_rt_free_block_ids": (i32, [vp, vp, i32, vp]),
        "vfl_rt_ref_count": (i32, [vp, i32, vp]),
        "vfl_rt_block_table": (i32, [vp, i32, vp, i32, vp]),
        "vfl_rt_required_new_blocks": (i32, [vp, vp, vp, i32, vp]),
        "vfl_rt_ensure_capacity": (i32, [vp, i32, i32, vp, vp]),
        "vfl_rt_fork": (i32, [vp, i32, i32]),
        "vfl_rt_deallocate": (i32, [vp, i32]),
        "vfl_rt_admit": (i32, [vp, i64, i32, vp]),
        "vfl_rt_num_running": (i32, [vp, vp]),
        "vfl_rt_prepare_step": (i32, [vp, vp, i32, vp]),
        "vfl_rt_pack_step": (i32, [vp, i32, vp, i64, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
        "vfl_rt_advance_greedy": (i32, [vp, ctypes.POINTER(DecodeRules), vp, i32, ctypes.POINTER(StepResult)]),
        "vfl_rt_advance_beam": (i32, [vp, ctypes.POINTER(DecodeRules), vp, vp, vp, i32, i32,
                                      ctypes.POINTER(StepResult)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def lib():
    """The loaded library (loaded once per process)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"vflorence_b200: CUDA library {LIB_PATH} is not built "
                        "(run `python -m vflorence_b200.build`)")
                L = ctypes.CDLL(LIB_PATH)
                _declare(L)
                if L.vfl_abi_version() != ABI_VERSION:
                    raise ImportError("vflorence_b200: library ABI version mismatch")
                _lib = L
    return _lib


def last_error() -> str:
    return lib().vfl_last_error_message().decode(errors="replace")


def check(status: int, what: str = "") -> None:
    """Raise VflError (ValueError-like statuses included) for a non-zero status."""
    if status != VFL_OK:
        L = lib()
        msg = L.vfl_last_error_message().decode(errors="replace")
        kind = L.vfl_status_string(status).decode()
        raise VflError(status, f"vflorence_b200{(' ' + what) if what else ''}: {kind}: {msg}")
