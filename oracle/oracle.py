"""ORACLE — test infrastructure only (never imported by the vflorence_b200 package).

ctypes wrapper around ``liboracle_paged.so`` (built from ``paged_ref.c`` by the Makefile in this
directory). Tensors are CPU ``torch`` tensors used as plain containers; every function here
mirrors one call site of the reference engine, named in ``paged_ref.c``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_paged.so")
_lib = None

F32, BF16 = 0, 1
_DTYPES = {torch.float32: F32, torch.bfloat16: BF16}


def build(force: bool = False) -> str:
    """Compile the oracle library with the Makefile beside this file; return its path."""
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
        os.path.join(_HERE, "paged_ref.c")
    ):
        subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.oracle_reshape_and_cache.restype = i64
        L.oracle_reshape_and_cache.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, i32, i64, i64, i64, i32]
        L.oracle_attention.restype = i64
        L.oracle_attention.argtypes = [vp, i64, vp, vp, i64, vp, i64, vp, vp, i32, vp, i64,
                                       i32, i32, i32, f32, i32, i32, i32]
        L.oracle_copy_blocks.restype = i64
        L.oracle_copy_blocks.argtypes = [vp, vp, i32, vp, i32, i64, i64]
        L.oracle_prepare_decode.restype = None
        L.oracle_prepare_decode.argtypes = [vp, i64, vp, i32, i32, vp, vp, vp]
        L.oracle_paged_slots.restype = None
        L.oracle_paged_slots.argtypes = [vp, i64, i32, i32, i32, vp]
        L.oracle_max_threads.restype = i32
        _lib = L
    return _lib


def max_threads() -> int:
    return lib().oracle_max_threads()


def _cpu(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.device.type != "cpu":
        raise ValueError(f"oracle: {name} must be a CPU tensor")
    return t


def _dtype(t: torch.Tensor) -> int:
    if t.dtype not in _DTYPES:
        raise ValueError(f"oracle: unsupported dtype {t.dtype}")
    return _DTYPES[t.dtype]


def reshape_and_cache(key, value, k_cache, v_cache, slot_mapping) -> int:
    """Scatter key/value rows [T, H, D] into the paged caches; returns skipped bad slots."""
    for name, t in (("key", key), ("value", value), ("k_cache", k_cache), ("v_cache", v_cache)):
        _cpu(t, name)
    assert key.stride(-1) == 1 and key.stride(-2) == key.shape[-1]
    assert value.stride(-1) == 1 and value.stride(-2) == value.shape[-1]
    assert k_cache.is_contiguous() and v_cache.is_contiguous()
    slots = _cpu(slot_mapping, "slot_mapping").to(torch.int64).contiguous()
    n, h, bs, d = k_cache.shape
    return lib().oracle_reshape_and_cache(
        key.data_ptr(), value.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), slots.data_ptr(),
        key.shape[0], h, d, bs, n, key.stride(0), value.stride(0), _dtype(k_cache))


def attention(query, k_cache, v_cache, output, query_start_loc, seq_lens, scale, causal,
              block_table, num_threads: int = 0) -> int:
    """Paged attention into ``output`` [T, H, D]; returns rows skipped for bad block ids."""
    for name, t in (("query", query), ("k_cache", k_cache), ("v_cache", v_cache), ("output", output)):
        _cpu(t, name)
    assert query.stride(-1) == 1 and query.stride(-2) == query.shape[-1]
    assert output.stride(-1) == 1 and output.stride(-2) == output.shape[-1]
    qsl = _cpu(query_start_loc, "query_start_loc").to(torch.int32).contiguous()
    lens = _cpu(seq_lens, "seq_lens").to(torch.int32).contiguous()
    table = _cpu(block_table, "block_table").to(torch.int32)
    if table.dim() != 2 or table.stride(1) != 1:
        table = table.contiguous()
    n, h, bs, d = k_cache.shape
    return lib().oracle_attention(
        query.data_ptr(), query.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), n,
        output.data_ptr(), output.stride(0), qsl.data_ptr(), lens.data_ptr(), lens.numel(),
        table.data_ptr(), table.stride(0) if table.shape[1] else 0, h, d, bs, float(scale),
        int(bool(causal)), _dtype(query), num_threads)


def copy_blocks(k_caches, v_caches, pairs) -> int:
    """Copy whole blocks src -> dst in every cache (gather then scatter)."""
    pairs_t = torch.as_tensor(pairs, dtype=torch.int64).reshape(-1, 2).contiguous()
    L = len(k_caches)
    kp = (ctypes.c_void_p * L)(*[c.data_ptr() for c in k_caches])
    vp = (ctypes.c_void_p * L)(*[c.data_ptr() for c in v_caches])
    c0 = k_caches[0]
    block_bytes = c0[0].numel() * c0.element_size()
    return lib().oracle_copy_blocks(kp, vp, L, pairs_t.data_ptr(), pairs_t.shape[0], c0.shape[0],
                                    block_bytes)


def prepare_decode(block_table, positions, block_size):
    """(slot_mapping int64, context_lens int32, query_start_loc int32) for one decode step."""
    table = block_table.to(torch.int32).contiguous()
    pos = positions.to(torch.int32).contiguous()
    b = pos.numel()
    slots = torch.empty(b, dtype=torch.int64)
    lens = torch.empty(b, dtype=torch.int32)
    qsl = torch.empty(b + 1, dtype=torch.int32)
    lib().oracle_prepare_decode(table.data_ptr(), table.stride(0) if table.dim() == 2 else 0,
                                pos.data_ptr(), b, block_size, slots.data_ptr(), lens.data_ptr(),
                                qsl.data_ptr())
    return slots, lens, qsl


def paged_slots(pages, seq_len, block_size):
    """Encoder slots of G requests of equal length from their pages [G, M]."""
    pages = pages.to(torch.int32).contiguous()
    out = torch.empty(pages.shape[0] * seq_len, dtype=torch.int64)
    lib().oracle_paged_slots(pages.data_ptr(), pages.stride(0), pages.shape[0], seq_len, block_size,
                             out.data_ptr())
    return out
