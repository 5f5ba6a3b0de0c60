"""The four ``vllm_cpu_attn`` functions the vflorence engine calls, on B200, plus the two ops
that sit beside them (copy-on-write block copies and the per-step metadata build).

Drop-in use: ``import vflorence_b200.paged_ops as vllm_cpu_attn``. Signatures and argument
meaning follow the call sites in vflorence (paths inside that project):

    get_isa                   vflorence/engine/model_runner.py:38
    get_scheduler_metadata    vflorence/layers/attention.py:18-29, model_runner.py:308-319
    reshape_and_cache         vflorence/layers/attention.py:55-57, model_runner.py:252-259
    attention_with_kv_cache   vflorence/layers/attention.py:61-72, :98-109
    copy_blocks               replaces ModelRunner._copy_blocks, model_runner.py:162-167
    prepare_decode            replaces the list building of ModelRunner._prepare, :290-306
    paged_slots               replaces the encoder slot arithmetic of _encode, :240-242

Differences a caller sees:
  * caches, queries, keys, values and outputs live on one CUDA device; a CPU one is an error
    (there is no CPU path). The small integer metadata may come from the host in the forms the
    reference builds them (``slot_mapping``, ``seq_lens``, ``query_start_loc``, block tables made
    by ``pad_sequence``; vflorence/layers/attention.py:9-39, model_runner.py:290-306): each such
    tensor is uploaded inside the call, one copy on the current stream (pinned ones with a wait
    for that copy, so the caller may reuse them at once). Device metadata costs no copy.
    ``get_scheduler_metadata`` reads its lengths on the host - pass host tensors (the engine has
    them), or it copies (and synchronises) once.
  * the metadata is a host int64 tensor holding a ``vfl_attention_plan``; pass the same device
    lengths to ``attention_with_kv_cache`` as were planned (longer ones are clamped and flagged).
  * several query rows of one request (``query_start_loc``) attend to the same pages, so beams
    sharing an encoder output can be one request: its pages are read once for all of them.
Everything is enqueued on the current CUDA stream; nothing synchronises.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N

HEAD_DIMS = frozenset({32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256, 512})
_DTYPES = {torch.float32: N.DTYPE_F32, torch.bfloat16: N.DTYPE_BF16}


def _dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise ValueError(f"vflorence_b200: dtype {dtype} is not supported (float32, bfloat16)") from None


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(name: str, t: torch.Tensor, device: torch.device | None = None) -> None:
    if not t.is_cuda:
        raise ValueError(f"vflorence_b200: {name} must be a CUDA tensor (got {t.device})")
    if device is not None and t.device != device:
        raise ValueError(f"vflorence_b200: {name} is on {t.device}, expected {device}")


def _require_dense_rows(name: str, t: torch.Tensor) -> None:
    """[tokens, heads, head_dim] with dense heads and elements (any token stride)."""
    if t.dim() != 3 or t.stride(2) != 1 or t.stride(1) != t.shape[2]:
        raise ValueError(f"vflorence_b200: {name} must be [tokens, heads, head_dim] with dense "
                         f"heads (got shape {tuple(t.shape)}, strides {t.stride()})")


def _on_device(name: str, t: torch.Tensor, device: torch.device) -> torch.Tensor:
    """Integer metadata on ``device``: a host tensor (the reference's form) is uploaded on the
    current stream - pageable memory is staged before the copy returns, pinned memory is waited
    for - so the caller may change or free its tensor after the call."""
    if t.device.type == "cpu":
        return t.to(device, non_blocking=not t.is_pinned())
    _require_cuda(name, t, device)
    return t


def _host_int32(t: torch.Tensor | None) -> torch.Tensor | None:
    if t is None:
        return None
    if t.device.type != "cpu":
        t = t.cpu()
    return t.to(torch.int32).contiguous()


# ------------------------------------------------------------------------------------- get_isa

def get_isa(dtype: torch.dtype, block_size: int, head_dim: int) -> str:
    """Kernel family tag for (dtype, block_size, head_dim): ``"sm100"``.

    Raises ValueError for a configuration the B200 kernels do not cover (the reference raises
    ValueError for an unsupported head_dim, vflorence/engine/model_runner.py:33-37).
    """
    buf = ctypes.create_string_buffer(16)
    st = N.lib().vfl_get_isa(_dtype_code(dtype), int(block_size), int(head_dim), buf, 16)
    if st != N.VFL_OK:
        raise ValueError(f"vflorence_b200: {N.last_error()}")
    return buf.value.decode()


# ------------------------------------------------------------------------ scheduler metadata

def row_tables_supported(dtype: torch.dtype, head_dim: int) -> bool:
    """Whether attention with per-row block tables is built for this shape (bf16, head_dim 64)."""
    return dtype == torch.bfloat16 and head_dim == 64


def row_tables_pay_off(groups: int, num_heads: int) -> bool:
    """Whether grouping beams (one CTA per request and head group instead of per row) keeps
    enough CTAs in flight: at least half a wave (148 SMs x 3 CTAs / 2). Measured on decode
    steps: 86 requests x 4 head groups 11 % faster than row by row, 64 x 3 even, 32 x 4 3-7 %
    slower."""
    head_groups = num_heads // 4 if num_heads % 4 == 0 else (num_heads // 2 if num_heads % 2 == 0 else num_heads)
    return groups * head_groups >= 148 * 3 // 2


def get_scheduler_metadata(num_reqs: int, num_heads: int, num_kv_heads: int, head_dim: int,
                           seq_lens: torch.Tensor, dtype: torch.dtype,
                           query_start_loc: torch.Tensor | None, causal: bool, isa: str,
                           block_size: int, row_tables: bool = False) -> torch.Tensor:
    """Launch plan for ``attention_with_kv_cache``: a host int64 tensor holding the plan struct.

    ``row_tables``: every query row has its own block table (the beams of a request, grouped
    by ``query_start_loc``, one length per request); bf16 with head_dim 64, not causal."""
    lens = _host_int32(seq_lens)
    if lens.numel() != num_reqs:
        raise ValueError(f"vflorence_b200: seq_lens has {lens.numel()} entries for {num_reqs} requests")
    qsl = _host_int32(query_start_loc)
    if qsl is not None and qsl.numel() != num_reqs + 1:
        raise ValueError("vflorence_b200: query_start_loc must have num_reqs + 1 entries")
    meta = torch.zeros(N.PLAN_BYTES // 8, dtype=torch.int64)
    plan = N.AttentionPlan.from_address(meta.data_ptr())
    if row_tables:
        if causal:
            raise ValueError("vflorence_b200: row_tables plans are not causal")
        if qsl is None:
            raise ValueError("vflorence_b200: row_tables plans need query_start_loc")
        st = N.lib().vfl_plan_attention_row_tables(int(num_reqs), int(num_heads), int(num_kv_heads), int(head_dim),
                                                   int(block_size), _dtype_code(dtype),
                                                   lens.data_ptr() if num_reqs else None, qsl.data_ptr(),
                                                   ctypes.byref(plan))
    else:
        st = N.lib().vfl_plan_attention(int(num_reqs), int(num_heads), int(num_kv_heads), int(head_dim),
                                        int(block_size), _dtype_code(dtype), int(bool(causal)),
                                        lens.data_ptr() if num_reqs else None,
                                        qsl.data_ptr() if qsl is not None else None, ctypes.byref(plan))
    N.check(st, "get_scheduler_metadata")
    return meta


SCHEDULE_ITEMS = 0     # one CTA per (request, head group, query chunk, split)
SCHEDULE_BALANCED = 1  # one persistent wave; equal runs of 16-token tiles per CTA


def set_schedule(metadata: torch.Tensor, schedule: int, min_tiles: int = 0) -> torch.Tensor:
    """Re-plan ``metadata`` (in place) for ``SCHEDULE_ITEMS`` or ``SCHEDULE_BALANCED`` (at least
    ``min_tiles`` 16-token tiles per CTA; 0: the default); returns it. ``ValueError`` when the
    plan cannot take that schedule."""
    plan = plan_of(metadata)
    st = N.lib().vfl_plan_attention_schedule(ctypes.byref(plan), int(schedule), int(min_tiles))
    if st != N.VFL_OK:
        raise ValueError(f"vflorence_b200: {N.last_error()}")
    return metadata


def plan_of(metadata: torch.Tensor) -> N.AttentionPlan:
    """View the plan struct stored in a metadata tensor (no copy; the view keeps the tensor's
    memory alive, so ``plan_of(get_scheduler_metadata(...))`` is safe)."""
    if (metadata.device.type != "cpu" or metadata.dtype != torch.int64 or not metadata.is_contiguous()
            or metadata.numel() * 8 < N.PLAN_BYTES):
        raise ValueError("vflorence_b200: scheduler_metadata must come from get_scheduler_metadata")
    plan = N.AttentionPlan.from_buffer(metadata.numpy())  # holds the array, which holds the tensor
    if plan.magic != N.PLAN_MAGIC:
        raise ValueError("vflorence_b200: scheduler_metadata must come from get_scheduler_metadata")
    return plan


# ------------------------------------------------------------------------- reshape_and_cache

def reshape_and_cache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                      v_cache: torch.Tensor, slot_mapping: torch.Tensor, isa: str | None = None) -> None:
    """``k_cache[s // bs, h, s % bs] = key[t, h]`` (same for value) for ``s = slot_mapping[t] >= 0``.
    ``slot_mapping`` may be a host tensor (uploaded inside the call)."""
    dev = k_cache.device
    for name, t in (("key", key), ("value", value), ("k_cache", k_cache), ("v_cache", v_cache)):
        _require_cuda(name, t, dev)
    slot_mapping = _on_device("slot_mapping", slot_mapping, dev)
    _require_dense_rows("key", key)
    _require_dense_rows("value", value)
    if key.shape != value.shape or key.dtype != k_cache.dtype or value.dtype != v_cache.dtype:
        raise ValueError("vflorence_b200: key/value shapes or dtypes do not match the caches")
    if k_cache.shape != v_cache.shape or k_cache.dim() != 4 or not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("vflorence_b200: caches must be contiguous [num_blocks, heads, block_size, head_dim]")
    n, h, bs, d = k_cache.shape
    if key.shape[1:] != (h, d):
        raise ValueError(f"vflorence_b200: key rows {tuple(key.shape[1:])} do not match the cache ({h}, {d})")
    if slot_mapping.dtype != torch.int64 or slot_mapping.dim() != 1 or slot_mapping.numel() != key.shape[0]:
        raise ValueError("vflorence_b200: slot_mapping must be int64 [num_tokens]")
    slots = slot_mapping if slot_mapping.is_contiguous() else slot_mapping.contiguous()
    st = N.lib().vfl_reshape_and_cache(key.data_ptr(), value.data_ptr(), k_cache.data_ptr(),
                                       v_cache.data_ptr(), slots.data_ptr(), key.shape[0], h, d, bs, n,
                                       key.stride(0), value.stride(0), _dtype_code(k_cache.dtype),
                                       _stream(dev))
    N.check(st, "reshape_and_cache")


# ------------------------------------------------------------------- attention_with_kv_cache

def _attention_checks(plan, query, k_cache, v_cache, output, query_start_loc, seq_lens, causal, block_table):
    """Checks shared by the attention entry points. Returns (device, pool blocks, workspace,
    query_start_loc, seq_lens, block_table) with the metadata on the device."""
    dev = k_cache.device
    for name, t in (("query", query), ("k_cache", k_cache), ("v_cache", v_cache), ("output", output)):
        _require_cuda(name, t, dev)
    query_start_loc = _on_device("query_start_loc", query_start_loc, dev)
    seq_lens = _on_device("seq_lens", seq_lens, dev)
    block_table = _on_device("block_table", block_table, dev)
    _require_dense_rows("query", query)
    _require_dense_rows("output", output)
    n, h, bs, d = k_cache.shape
    if (plan.num_heads, plan.head_dim, plan.block_size, plan.dtype) != (h, d, bs, _dtype_code(k_cache.dtype)):
        raise ValueError("vflorence_b200: scheduler_metadata was planned for another cache shape or dtype")
    if bool(plan.causal) != bool(causal):
        raise ValueError("vflorence_b200: scheduler_metadata was planned with another causal flag")
    if query.dtype != k_cache.dtype or output.dtype != k_cache.dtype or v_cache.shape != k_cache.shape:
        raise ValueError("vflorence_b200: query/output/cache dtypes or cache shapes differ")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("vflorence_b200: caches must be contiguous")
    if query.shape != output.shape or query.shape[1:] != (h, d) or query.shape[0] < plan.total_q:
        raise ValueError("vflorence_b200: query/output must be [num_tokens >= planned rows, heads, head_dim]")
    if (query_start_loc.dtype != torch.int32 or seq_lens.dtype != torch.int32 or block_table.dtype != torch.int32
            or block_table.dim() != 2 or block_table.stride(1) != 1):
        raise ValueError("vflorence_b200: query_start_loc, seq_lens and block_table must be int32 "
                         "(block_table [num_reqs, cols] with unit column stride)")
    if seq_lens.numel() != plan.num_reqs or query_start_loc.numel() != plan.num_reqs + 1 \
            or block_table.shape[0] < (plan.total_q if plan.row_tables else plan.num_reqs):
        raise ValueError("vflorence_b200: metadata planned for a different number of requests "
                         "(with row tables, block_table holds one row per query row)")
    ws = None
    if plan.workspace_bytes > 0:
        ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=dev)
    return dev, n, ws, query_start_loc, seq_lens, block_table


def attention_with_kv_cache(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            output: torch.Tensor, query_start_loc: torch.Tensor,
                            seq_lens: torch.Tensor, scale: float, causal: bool,
                            block_table: torch.Tensor, scheduler_metadata: torch.Tensor) -> None:
    """``output = softmax(scale * q K^T) V`` per request over its paged tokens (writes ``output``).
    ``query_start_loc``, ``seq_lens`` and ``block_table`` may be host tensors (uploaded inside the
    call), as the reference passes them."""
    plan = plan_of(scheduler_metadata)
    dev, n, ws, query_start_loc, seq_lens, block_table = _attention_checks(
        plan, query, k_cache, v_cache, output, query_start_loc, seq_lens, causal, block_table)
    st = N.lib().vfl_attention_with_kv_cache(
        ctypes.byref(plan), query.data_ptr(), query.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), n,
        output.data_ptr(), output.stride(0), query_start_loc.data_ptr(), seq_lens.data_ptr(),
        block_table.data_ptr(), block_table.stride(0), block_table.shape[1], float(scale),
        ws.data_ptr() if ws is not None else None, plan.workspace_bytes if ws is not None else 0,
        _stream(dev))
    N.check(st, "attention_with_kv_cache")


def attention_append_supported(scheduler_metadata: torch.Tensor) -> bool:
    """Whether ``attention_with_kv_cache_append`` takes this plan: one new token per query row,
    and either one row per request (any dtype and head_dim), or with the tensor-core kernel
    (bf16, head_dim 64) at most 8 causal rows per request or rows with their own tables."""
    return bool(N.lib().vfl_attention_append_supported(ctypes.byref(plan_of(scheduler_metadata))))


def attention_with_kv_cache_append(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                                   k_cache: torch.Tensor, v_cache: torch.Tensor, output: torch.Tensor,
                                   slot_mapping: torch.Tensor, query_start_loc: torch.Tensor,
                                   seq_lens: torch.Tensor, scale: float, causal: bool, block_table: torch.Tensor,
                                   scheduler_metadata: torch.Tensor) -> None:
    """``reshape_and_cache(key, value, k_cache, v_cache, slot_mapping)`` then
    ``attention_with_kv_cache(...)`` in one launch (vflorence/layers/attention.py:55-72): query row
    t's new key / value rows go to ``slot_mapping[t]`` before the attention reads them. Each
    row's new token is the newest position of its sequence, or for causal rows the successive
    positions ending there, in a block no other row of the call holds. Plans for which
    ``attention_append_supported`` is False raise VflError."""
    plan = plan_of(scheduler_metadata)
    dev, n, ws, query_start_loc, seq_lens, block_table = _attention_checks(
        plan, query, k_cache, v_cache, output, query_start_loc, seq_lens, causal, block_table)
    for name, t in (("key", key), ("value", value)):
        _require_cuda(name, t, dev)
    slot_mapping = _on_device("slot_mapping", slot_mapping, dev)
    _require_dense_rows("key", key)
    _require_dense_rows("value", value)
    if key.shape != value.shape or key.shape[1:] != query.shape[1:] or key.shape[0] < plan.total_q \
            or key.dtype != k_cache.dtype or value.dtype != k_cache.dtype:
        raise ValueError("vflorence_b200: key/value must be [query rows, heads, head_dim] of the cache dtype")
    if slot_mapping.dtype != torch.int64 or slot_mapping.dim() != 1 or slot_mapping.numel() < plan.total_q \
            or not slot_mapping.is_contiguous():
        raise ValueError("vflorence_b200: slot_mapping must be contiguous int64 [query rows]")
    st = N.lib().vfl_attention_with_kv_cache_append(
        ctypes.byref(plan), query.data_ptr(), query.stride(0), key.data_ptr(), key.stride(0), value.data_ptr(),
        value.stride(0), slot_mapping.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), n, output.data_ptr(),
        output.stride(0), query_start_loc.data_ptr(), seq_lens.data_ptr(), block_table.data_ptr(),
        block_table.stride(0), block_table.shape[1], float(scale),
        ws.data_ptr() if ws is not None else None, plan.workspace_bytes if ws is not None else 0,
        _stream(dev))
    N.check(st, "attention_with_kv_cache_append")


# ------------------------------------------------------------------------------- copy_blocks

def check_copy_pairs(pairs, num_blocks: int) -> list[tuple[int, int]]:
    """Validate copy-on-write pairs on the host: in range, unique destinations, and no block
    both read and written (the gather-then-scatter meaning of index_select + index_copy_)."""
    pairs = [(int(s), int(d)) for s, d in pairs]
    srcs = {s for s, _ in pairs}
    dsts = [d for _, d in pairs]
    for s, d in pairs:
        if not (0 <= s < num_blocks and 0 <= d < num_blocks):
            raise ValueError(f"vflorence_b200: copy pair ({s}, {d}) outside [0, {num_blocks})")
    if len(set(dsts)) != len(dsts):
        raise ValueError("vflorence_b200: copy_blocks destinations must be unique")
    if srcs.intersection(dsts):
        raise ValueError("vflorence_b200: copy_blocks sources and destinations must be disjoint")
    return pairs


def check_copy_pairs_array(pairs, num_blocks: int) -> None:
    """``check_copy_pairs`` for an integer [P, 2] numpy array (vectorised)."""
    if pairs.ndim != 2 or pairs.shape[1] != 2:
        raise ValueError("vflorence_b200: copy pairs must be a [P, 2] array")
    if len(pairs) == 0:
        return
    if pairs.min() < 0 or pairs.max() >= num_blocks:
        raise ValueError(f"vflorence_b200: a copy pair lies outside [0, {num_blocks})")
    src, dst = pairs[:, 0], pairs[:, 1]
    if np.unique(dst).size != dst.size:
        raise ValueError("vflorence_b200: copy_blocks destinations must be unique")
    if np.intersect1d(src, dst).size:
        raise ValueError("vflorence_b200: copy_blocks sources and destinations must be disjoint")


class CopyBlocksTarget:
    """A fixed set of per-layer K/V caches checked once for copy_blocks, with the pointer arrays
    the launches take (an engine's pools do not change between steps)."""

    def __init__(self, k_caches, v_caches):
        k_caches, v_caches = list(k_caches), list(v_caches)
        if len(k_caches) != len(v_caches) or not k_caches:
            raise ValueError("vflorence_b200: copy_blocks needs matching, non-empty K and V cache lists")
        c0 = k_caches[0]
        self.device = dev = c0.device
        for c in k_caches + v_caches:
            _require_cuda("cache", c, dev)
            if c.shape != c0.shape or c.dtype != c0.dtype or not c.is_contiguous():
                raise ValueError("vflorence_b200: copy_blocks caches must share one contiguous shape and dtype")
        self.caches = (k_caches, v_caches)  # keeps the pools alive while the pointers are held
        self.num_blocks = c0.shape[0]
        self.block_bytes = c0[0].numel() * c0.element_size()
        self.chunks = []
        for start in range(0, len(k_caches), N.MAX_COPY_LAYERS):
            ks, vs = k_caches[start:start + N.MAX_COPY_LAYERS], v_caches[start:start + N.MAX_COPY_LAYERS]
            self.chunks.append(((ctypes.c_void_p * len(ks))(*[c.data_ptr() for c in ks]),
                                (ctypes.c_void_p * len(vs))(*[c.data_ptr() for c in vs]), len(ks)))

    def launch(self, pairs_t: torch.Tensor, num_pairs: int) -> None:
        """Copy ``num_pairs`` (src, dst) rows of the device int64 tensor ``pairs_t`` [>= P, 2]."""
        if num_pairs == 0:
            return
        lib, stream = N.lib(), _stream(self.device)
        for kp, vp, n in self.chunks:
            st = lib.vfl_copy_blocks(kp, vp, n, pairs_t.data_ptr(), num_pairs, self.num_blocks, self.block_bytes,
                                     stream)
            N.check(st, "copy_blocks")


def copy_blocks(k_caches, v_caches, block_pairs) -> None:
    """For every layer: ``k_caches[l][dst] = k_caches[l][src]`` (and V) for each (src, dst).

    ``block_pairs`` is a list of (src, dst) (validated on the host and uploaded) or a device int64
    tensor [P, 2] (validated by the kernel only: out-of-range pairs are skipped and flagged).
    One launch covers all layers and pairs. ``k_caches`` may also be a CopyBlocksTarget (then
    ``v_caches`` is ignored), which skips re-checking the caches.
    """
    target = k_caches if isinstance(k_caches, CopyBlocksTarget) else CopyBlocksTarget(k_caches, v_caches)
    dev = target.device
    if isinstance(block_pairs, torch.Tensor):
        _require_cuda("block_pairs", block_pairs, dev)
        pairs_t = block_pairs.to(torch.int64).reshape(-1, 2).contiguous()
    else:
        pairs = check_copy_pairs(block_pairs, target.num_blocks)
        if not pairs:
            return
        pairs_t = torch.tensor(pairs, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
    target.launch(pairs_t, pairs_t.shape[0])


# ---------------------------------------------------------------------------- step metadata

def prepare_decode(block_table: torch.Tensor, positions: torch.Tensor, block_size: int,
                   slot_mapping: torch.Tensor, context_lens: torch.Tensor,
                   query_start_loc: torch.Tensor) -> None:
    """Fill one decode step's slot mapping (int64), context lengths and query_start_loc (int32)
    from the padded block table and each sequence's position (= cached tokens)."""
    dev = block_table.device
    for name, t in (("block_table", block_table), ("positions", positions), ("slot_mapping", slot_mapping),
                    ("context_lens", context_lens), ("query_start_loc", query_start_loc)):
        _require_cuda(name, t, dev)
    b = positions.numel()
    if (block_table.dtype != torch.int32 or positions.dtype != torch.int32 or block_table.dim() != 2
            or block_table.stride(1) != 1 or block_table.shape[0] < b or not positions.is_contiguous()):
        raise ValueError("vflorence_b200: prepare_decode wants int32 block_table [B, M] and positions [B]")
    if (slot_mapping.dtype != torch.int64 or context_lens.dtype != torch.int32
            or query_start_loc.dtype != torch.int32 or slot_mapping.numel() < b
            or context_lens.numel() < b or query_start_loc.numel() < b + 1):
        raise ValueError("vflorence_b200: prepare_decode output dtypes or sizes are wrong")
    st = N.lib().vfl_prepare_decode(block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
                                    positions.data_ptr(), b, int(block_size), slot_mapping.data_ptr(),
                                    context_lens.data_ptr(), query_start_loc.data_ptr(), _stream(dev))
    N.check(st, "prepare_decode")


def add_layernorm_supported(dtype: torch.dtype, hidden_dim: int) -> bool:
    """Whether the fused residual add + LayerNorm is built for this dtype and row width."""
    return dtype in (torch.float32, torch.bfloat16) and bool(
        N.lib().vfl_add_layernorm_supported(_dtype_code(dtype), int(hidden_dim)))


def add_layernorm(h: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                  eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """``LayerNorm(h + x) * weight + bias`` over the last dimension of [rows, d] tensors, in one
    launch - the post-norm residual of the decoder (vflorence/models/bart.py:192-201). ``h + x``
    is rounded to the dtype first, as ``h + x`` is; statistics in fp32. Returns ``out`` (new
    unless given; it may be ``h`` or ``x``)."""
    dev = h.device
    for name, t in (("h", h), ("x", x), ("weight", weight)):
        _require_cuda(name, t, dev)
    if h.dim() != 2 or x.shape != h.shape or h.stride(1) != 1 or x.stride(1) != 1:
        raise ValueError("vflorence_b200: add_layernorm wants h and x [rows, d] with unit column stride")
    rows, d = h.shape
    if x.dtype != h.dtype or weight.dtype != h.dtype or weight.shape != (d,) or not weight.is_contiguous():
        raise ValueError("vflorence_b200: add_layernorm weight must be contiguous [d] of the rows' dtype")
    if bias is not None:
        _require_cuda("bias", bias, dev)
        if bias.dtype != h.dtype or bias.shape != (d,) or not bias.is_contiguous():
            raise ValueError("vflorence_b200: add_layernorm bias must be contiguous [d] of the rows' dtype")
    if out is None:
        out = torch.empty_like(h, memory_format=torch.contiguous_format)
    elif out.shape != h.shape or out.dtype != h.dtype or out.stride(1) != 1 or out.device != dev:
        raise ValueError("vflorence_b200: add_layernorm out must match h")
    st = N.lib().vfl_add_layernorm(h.data_ptr(), h.stride(0), x.data_ptr(), x.stride(0), weight.data_ptr(),
                                   None if bias is None else bias.data_ptr(), out.data_ptr(), out.stride(0),
                                   rows, d, float(eps), _dtype_code(h.dtype), _stream(dev))
    N.check(st, "add_layernorm")
    return out


def kv_proj_supported(dtype: torch.dtype, hidden_dim: int, num_heads: int, head_dim: int) -> bool:
    """Whether the fused projection + page write is built for this shape (bf16 tensor cores)."""
    return (dtype == torch.bfloat16 and hidden_dim % 64 == 0 and head_dim % 32 == 0
            and (2 * num_heads * head_dim) % 128 == 0)


def kv_proj_paged(hidden: torch.Tensor, w_kv: torch.Tensor, bias: torch.Tensor | None, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """``kv = hidden @ w_kv.T (+ bias)`` written straight into the paged caches: row t's first
    half (k) and second half (v), split into heads, go to ``slot_mapping[t]`` (negative: skip).
    hidden [T, hidden_dim] bf16 (unit column stride), w_kv [2 * H * D, hidden_dim] contiguous,
    caches [num_blocks, H, block_size, D] bf16, slot_mapping int64 [T]."""
    dev = k_cache.device
    for name, t in (("hidden", hidden), ("w_kv", w_kv), ("k_cache", k_cache), ("v_cache", v_cache),
                    ("slot_mapping", slot_mapping)):
        _require_cuda(name, t, dev)
    n, h, bs, d = k_cache.shape
    if (hidden.dtype != torch.bfloat16 or w_kv.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16
            or v_cache.shape != k_cache.shape or v_cache.dtype != k_cache.dtype):
        raise ValueError("vflorence_b200: kv_proj_paged is built for bfloat16")
    if hidden.dim() != 2 or hidden.stride(1) != 1 or not w_kv.is_contiguous() or w_kv.shape != (2 * h * d, hidden.shape[1]):
        raise ValueError("vflorence_b200: kv_proj_paged wants hidden [T, K] (unit column stride) and w_kv [2*H*D, K]")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("vflorence_b200: caches must be contiguous")
    if bias is not None:
        _require_cuda("bias", bias, dev)
        if bias.dtype != torch.bfloat16 or bias.numel() != 2 * h * d or not bias.is_contiguous():
            raise ValueError("vflorence_b200: kv_proj_paged bias must be contiguous bf16 [2*H*D]")
    if slot_mapping.dtype != torch.int64 or slot_mapping.numel() < hidden.shape[0] or not slot_mapping.is_contiguous():
        raise ValueError("vflorence_b200: slot_mapping must be contiguous int64 [T]")
    st = N.lib().vfl_kv_proj_paged(hidden.data_ptr(), hidden.stride(0), w_kv.data_ptr(),
                                   None if bias is None else bias.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                   slot_mapping.data_ptr(), hidden.shape[0], hidden.shape[1], h, d, bs, n,
                                   _stream(dev))
    N.check(st, "kv_proj_paged")


def paged_slots(pages: torch.Tensor, seq_len: int, block_size: int) -> torch.Tensor:
    """Slots of ``seq_len`` tokens for each row of ``pages`` [G, M] (int64 [G * seq_len])."""
    _require_cuda("pages", pages)
    if pages.dtype != torch.int32 or pages.dim() != 2 or pages.stride(1) != 1:
        raise ValueError("vflorence_b200: pages must be int32 [G, M] with unit column stride")
    out = torch.empty(pages.shape[0] * int(seq_len), dtype=torch.int64, device=pages.device)
    st = N.lib().vfl_paged_slots(pages.data_ptr(), pages.stride(0), pages.shape[1], pages.shape[0],
                                 int(seq_len), int(block_size), out.data_ptr(), _stream(pages.device))
    N.check(st, "paged_slots")
    return out


# ---------------------------------------------------------------------- candidate selection
MAX_TOPK = 64


def row_topk(scores: torch.Tensor, k: int, log_softmax: bool = False, row_offset: torch.Tensor | None = None,
             out: tuple[torch.Tensor, torch.Tensor] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Each row's best ``k`` entries of a [rows, vocab] float32/bfloat16 matrix (unit column
    stride), as log-probs when ``log_softmax``, plus ``row_offset`` (float32 [rows]) when given:
    (values float32 [rows, k], indices int32 [rows, k]), value descending, ties by lower index."""
    _require_cuda("scores", scores)
    dev = scores.device
    if scores.dim() != 2 or scores.stride(1) != 1:
        raise ValueError("vflorence_b200: row_topk wants a [rows, vocab] matrix with unit column stride")
    rows, vocab = scores.shape
    if row_offset is not None:
        _require_cuda("row_offset", row_offset, dev)
        if row_offset.dtype != torch.float32 or row_offset.numel() < rows or not row_offset.is_contiguous():
            raise ValueError("vflorence_b200: row_offset must be contiguous float32 [rows]")
    if out is None:
        out = (torch.empty(rows, k, dtype=torch.float32, device=dev), torch.empty(rows, k, dtype=torch.int32, device=dev))
    values, indices = out
    lib = N.lib()
    ws_bytes = lib.vfl_row_topk_workspace_size(rows, vocab, int(k)) if 1 <= k <= vocab else 0
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
    st = lib.vfl_row_topk(scores.data_ptr(), _dtype_code(scores.dtype), rows, vocab,
                          scores.stride(0) if rows > 1 else vocab, int(bool(log_softmax)),
                          None if row_offset is None else row_offset.data_ptr(), int(k), values.data_ptr(),
                          indices.data_ptr(), None if ws is None else ws.data_ptr(), ws_bytes, _stream(dev))
    N.check(st, "row_topk")
    return values, indices


def beam_merge(values: torch.Tensor, indices: torch.Tensor, groups: torch.Tensor, ranks: torch.Tensor,
               num_groups: int, keep: int) -> torch.Tensor:
    """Per-request merge of ``row_topk`` candidates: int32 [3, num_groups, keep] (row, token,
    float32 bits of the value; row -1 pads). ``groups``/``ranks``: int32 [rows] on the device."""
    dev = values.device
    for name, t in (("values", values), ("indices", indices), ("groups", groups), ("ranks", ranks)):
        _require_cuda(name, t, dev)
        if not t.is_contiguous():
            raise ValueError(f"vflorence_b200: beam_merge {name} must be contiguous")
    if (values.dtype != torch.float32 or indices.dtype != torch.int32 or groups.dtype != torch.int32
            or ranks.dtype != torch.int32 or values.shape != indices.shape or values.dim() != 2):
        raise ValueError("vflorence_b200: beam_merge dtypes or shapes are wrong")
    rows, k = values.shape
    out = torch.empty(3, num_groups, keep, dtype=torch.int32, device=dev)
    st = N.lib().vfl_beam_merge(values.data_ptr(), indices.data_ptr(), rows, k, groups.data_ptr(), ranks.data_ptr(),
                                int(num_groups), int(keep), out.data_ptr(), _stream(dev))
    N.check(st, "beam_merge")
    return out


def fork_token_rows(tokens: torch.Tensor, born: torch.Tensor) -> None:
    """Beam children's token rows in one launch: ``tokens[child] = tokens[parent]`` with
    ``tokens[child, pos] = token`` for each column of ``born`` (device int32 [4, n]: parents,
    children, positions, tokens) - Sequence.fork (vflorence/engine/sequence.py:53-55). No child
    may be a parent in the same call."""
    dev = tokens.device
    _require_cuda("tokens", tokens, dev)
    _require_cuda("born", born, dev)
    if tokens.dtype != torch.int32 or tokens.dim() != 2 or tokens.stride(1) != 1:
        raise ValueError("vflorence_b200: tokens must be int32 [rows, width] with unit column stride")
    if born.dtype != torch.int32 or born.dim() != 2 or born.shape[0] != 4 or not born.is_contiguous():
        raise ValueError("vflorence_b200: born must be contiguous int32 [4, n]")
    st = N.lib().vfl_fork_token_rows(tokens.data_ptr(), tokens.stride(0), tokens.shape[0], tokens.shape[1],
                                     born.data_ptr(), born.shape[1], _stream(dev))
    N.check(st, "fork_token_rows")


def read_device_errors(device: torch.device | int | None = None, clear: bool = True) -> int:
    """VFL_DEVERR_* bits the kernels raised on ``device`` since the last clear (synchronises)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index or 0))
    bits = ctypes.c_uint(0)
    with torch.cuda.device(dev):
        st = N.lib().vfl_read_device_errors(ctypes.byref(bits), int(bool(clear)), _stream(dev))
    N.check(st, "read_device_errors")
    return bits.value


def check_bounded_wait(limit_ns: int, producer_arrives: bool = False,
                       device: torch.device | int | None = None) -> None:
    """Run the bounded shared-memory wait of the pipelined kernels on its own (one CTA) on the
    current stream: without the producer's arrival it gives up after ``limit_ns`` and raises
    VFL_DEVERR_TIMEOUT in the device error word (read it with ``read_device_errors``, which also
    clears it; attention launches exit at once while the bit is set)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index or 0))
    with torch.cuda.device(dev):
        st = N.lib().vfl_check_bounded_wait(int(bool(producer_arrives)), int(limit_ns), _stream(dev))
    N.check(st, "check_bounded_wait")


# ------------------------------------------------------------------------------ decode_linear

_ACTS = {None: 0, "gelu": 1}


def decode_linear_supported(dtype: torch.dtype, rows: int, n: int, k: int) -> bool:
    """Whether ``decode_linear`` is built for this layer: float32, 1..16 rows, n a multiple of 32,
    k a multiple of 128."""
    if dtype != torch.float32:
        return False
    return bool(N.lib().vfl_decode_linear_supported(N.DTYPE_F32, int(rows), int(n), int(k)))


def decode_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                  activation: str | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``act(x @ weight.T + bias)`` for the few rows of a decode step (torch.nn.Linear's layout,
    float32): one weight-streaming launch, bias and the exact GELU fused. Returns ``out`` (a new
    [rows, n] tensor when None)."""
    dev = weight.device
    _require_cuda("x", x, dev)
    _require_cuda("weight", weight, dev)
    if activation not in _ACTS:
        raise ValueError(f"vflorence_b200: decode_linear activation {activation!r} (None or 'gelu')")
    if x.dim() != 2 or weight.dim() != 2 or x.shape[1] != weight.shape[1] or x.stride(1) != 1 \
            or not weight.is_contiguous():
        raise ValueError("vflorence_b200: decode_linear takes x [rows, k] (unit column stride) and a "
                         "contiguous weight [n, k]")
    if x.dtype != weight.dtype or (bias is not None and (bias.dtype != weight.dtype or bias.shape != (weight.shape[0],)
                                                        or not bias.is_contiguous())):
        raise ValueError("vflorence_b200: decode_linear x, weight and bias must share one dtype; bias [n]")
    if bias is not None:
        _require_cuda("bias", bias, dev)
    rows, k = x.shape
    n = weight.shape[0]
    if out is None:
        out = torch.empty(rows, n, dtype=x.dtype, device=dev)
    elif out.shape != (rows, n) or out.dtype != x.dtype or out.stride(1) != 1:
        raise ValueError("vflorence_b200: decode_linear out must be [rows, n] with unit column stride")
    st = N.lib().vfl_decode_linear(x.data_ptr(), x.stride(0), weight.data_ptr(),
                                   bias.data_ptr() if bias is not None else None, out.data_ptr(), out.stride(0),
                                   rows, n, k, _dtype_code(x.dtype), _ACTS[activation], _stream(dev))
    N.check(st, "decode_linear")
    return out
