"""Device-resident KV state of the decoder: the parts of vflorence's ``ModelRunner`` that own the
paged path (vflorence/engine/model_runner.py), on one CUDA device.

    allocate_kv_cache   model_runner.py:62-100   per-layer self and cross pools [N, H, bs, D]
    copy_blocks         model_runner.py:162-167  copy-on-write pairs, all layers, one launch
    CrossPageAllocator, page_requests / write_encoder_kv / project_encoder_kv / clear_request / reset
                        model_runner.py:169-177, :232-259, :261-271
    prepare_decode      model_runner.py:273-341  one pinned upload + one kernel per step
    stage_cross         model_runner.py:320-327  memoised on the batch's request ids

The pools are separate tensors per layer (as in the reference), zero-filled once. The kernels
never read past a sequence's length, so the zero fill is for state parity only.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import attention, paged_ops


def pack_decode_step(block_tables, positions) -> np.ndarray:
    """One int32 host buffer for a decode step: the block tables zero-padded to a rectangle
    [B, max_blocks] (vflorence/engine/model_runner.py:302-304), then the positions [B]."""
    b = len(positions)
    width = max(len(t) for t in block_tables)
    host = np.zeros(b * width + b, dtype=np.int32)
    tables = host[: b * width].reshape(b, width)
    for i, t in enumerate(block_tables):
        tables[i, : len(t)] = t
    host[b * width:] = positions
    return host


class CrossPageAllocator:
    """Encoder K/V pages of the fixed cross pool: a request takes its pages from the END of the
    free list and returns them to the end when it finishes (vflorence/engine/model_runner.py:
    169-177, :261-271). Host bookkeeping only."""

    def __init__(self, num_pages: int):
        self.num_pages = num_pages
        self.reset()

    def reset(self) -> None:
        self.pages: dict[int, tuple[torch.Tensor, int]] = {}
        self.free = list(range(self.num_pages))

    def allocate(self, num_pages: int) -> list[int]:
        if num_pages > len(self.free):
            raise RuntimeError("encoder K/V pool is full; increase max_num_seqs or max_encoder_len")
        taken = self.free[len(self.free) - num_pages:]
        del self.free[len(self.free) - num_pages:]
        return taken

    def assign(self, request_ids, enc_len: int, block_size: int) -> torch.Tensor:
        """Pages for a same-length group: int32 [G, ceil(enc_len / block_size)] (host)."""
        per_req = -(-enc_len // block_size)
        pages = torch.tensor(self.allocate(len(request_ids) * per_req), dtype=torch.int32)
        pages = pages.view(len(request_ids), per_req)
        for rid, row in zip(request_ids, pages):
            self.pages[rid] = (row, enc_len)
        return pages

    def release(self, request_id: int) -> None:
        pages, _ = self.pages.pop(request_id, ((), 0))
        self.free.extend(int(p) for p in pages)


@dataclass
class DecodeStep:
    """Device tensors of one decode step (what ``set_context`` publishes)."""

    positions: torch.Tensor        # int32 [B]
    slot_mapping: torch.Tensor     # int64 [B]
    context_lens: torch.Tensor     # int32 [B]
    block_tables: torch.Tensor     # int32 [B, max_blocks]
    query_start_loc: torch.Tensor  # int32 [B + 1]
    self_metadata: torch.Tensor    # host plan
    context_lens_host: torch.Tensor


class PagedKVCache:
    def __init__(self, *, num_layers: int, num_heads: int, head_dim: int, block_size: int,
                 num_blocks: int, num_cross_blocks: int, dtype: torch.dtype,
                 device: torch.device | str = "cuda"):
        self.isa = paged_ops.get_isa(dtype, block_size, head_dim)
        self.num_layers, self.num_heads, self.head_dim = num_layers, num_heads, head_dim
        self.block_size, self.num_blocks, self.num_cross_blocks = block_size, num_blocks, num_cross_blocks
        self.dtype = dtype
        self.device = torch.device(device)
        shape = (num_blocks, num_heads, block_size, head_dim)
        cross = (num_cross_blocks, num_heads, block_size, head_dim)
        z = lambda s: torch.zeros(s, dtype=dtype, device=self.device)  # noqa: E731
        self.k_caches = [z(shape) for _ in range(num_layers)]
        self.v_caches = [z(shape) for _ in range(num_layers)]
        self.cross_k_caches = [z(cross) for _ in range(num_layers)]
        self.cross_v_caches = [z(cross) for _ in range(num_layers)]
        self.cross = CrossPageAllocator(num_cross_blocks)
        self._cross_key = None
        self._cross_staged = None
        self._pairs_host = self._pairs_dev = None
        self._copy = None  # CopyBlocksTarget over the self-attention pools, made on first use

    # ----------------------------------------------------------------------------- binding
    def bind(self, decoder_layers) -> None:
        """Attach the pools to decoder layers (``self_attn`` / ``encoder_attn`` modules)."""
        for i, layer in enumerate(decoder_layers):
            layer.self_attn.k_cache, layer.self_attn.v_cache = self.k_caches[i], self.v_caches[i]
            layer.encoder_attn.k_cache = self.cross_k_caches[i]
            layer.encoder_attn.v_cache = self.cross_v_caches[i]

    @property
    def nbytes(self) -> int:
        return sum(t.nbytes for t in self.k_caches + self.v_caches + self.cross_k_caches + self.cross_v_caches)

    # ------------------------------------------------------------------------ copy-on-write
    def copy_blocks(self, copies, checked: bool = False) -> None:
        """Copy whole self-attention blocks src -> dst in every layer (before the step's append).
        ``copies``: (src, dst) pairs, a list or an integer [P, 2] array (uploaded through one
        reused pinned buffer). ``checked``: the pairs come from the native runtime, which only
        makes in-range pairs with distinct destinations disjoint from the sources (the kernel
        still skips and flags out-of-range pairs); others are checked on the host."""
        if isinstance(copies, np.ndarray):
            pairs = np.asarray(copies, dtype=np.int64).reshape(-1, 2)
            P = len(pairs)
            if P == 0:
                return
            if not checked:
                paged_ops.check_copy_pairs_array(pairs, self.num_blocks)
            if self._pairs_host is None or self._pairs_host.numel() < 2 * P:
                self._pairs_host = torch.zeros(max(2 * P, 1024), dtype=torch.int64).pin_memory()
                self._pairs_dev = torch.zeros_like(self._pairs_host, device=self.device)
            self._pairs_host.numpy()[: 2 * P] = pairs.reshape(-1)
            dev = self._pairs_dev[: 2 * P]
            dev.copy_(self._pairs_host[: 2 * P], non_blocking=True)
            self._copy_target().launch(dev, P)
        elif copies:
            paged_ops.copy_blocks(self._copy_target(), None, copies)

    def _copy_target(self) -> paged_ops.CopyBlocksTarget:
        if self._copy is None:  # the pools are checked once, not per step
            self._copy = paged_ops.CopyBlocksTarget(self.k_caches, self.v_caches)
        return self._copy

    # ------------------------------------------------------------------------ encoder pages
    def page_requests(self, request_ids, enc_len: int) -> torch.Tensor:
        """Give each request of a same-length group its pages; returns the group's slots
        (int64 [G * enc_len], device), token t of request g at ``pages[g, t // bs] * bs + t % bs``."""
        pages = self.cross.assign(request_ids, enc_len, self.block_size)
        pages_dev = pages.pin_memory().to(self.device, non_blocking=True)
        return paged_ops.paged_slots(pages_dev, enc_len, self.block_size)

    def write_encoder_kv(self, layer: int, key: torch.Tensor, value: torch.Tensor, slots: torch.Tensor) -> None:
        """Store one layer's encoder K/V rows [G * enc_len, H, D] at ``slots``."""
        paged_ops.reshape_and_cache(key, value, self.cross_k_caches[layer], self.cross_v_caches[layer],
                                    slots, isa=self.isa)

    def project_encoder_kv(self, layer: int, hidden: torch.Tensor, w_kv: torch.Tensor, b_kv: torch.Tensor | None,
                           slots: torch.Tensor) -> None:
        """One layer's encoder K/V projected from ``hidden`` [G * S, d_model] and written at
        ``slots`` in one launch (bf16 tensor cores; vfl_kv_proj_paged)."""
        paged_ops.kv_proj_paged(hidden, w_kv, b_kv, self.cross_k_caches[layer], self.cross_v_caches[layer], slots)

    def clear_request(self, request_id: int) -> None:
        self.cross.release(request_id)
        self._cross_key = self._cross_staged = None

    def reset(self) -> None:
        self.cross.reset()
        self._cross_key = self._cross_staged = None

    # --------------------------------------------------------------------------- per step
    def prepare_decode(self, block_tables, positions) -> DecodeStep:
        """Upload one step's block tables and positions (one pinned copy) and derive the slot
        mapping, context lengths and query_start_loc on the device."""
        b = len(positions)
        width = max(len(t) for t in block_tables)
        host = torch.from_numpy(pack_decode_step(block_tables, positions)).pin_memory()
        return self.prepare_decode_host(host, b, width)

    def prepare_decode_host(self, host: torch.Tensor, b: int, width: int) -> DecodeStep:
        """``prepare_decode`` from a pinned int32 host buffer that already holds the block
        tables [b, width] followed by the positions [b]."""
        pos = host.numpy()[b * width: b * width + b]
        dev = host[: b * width + b].to(self.device, non_blocking=True)
        tables_dev = dev[: b * width].view(b, width)
        pos_dev = dev[b * width:]
        slot_mapping = torch.empty(b, dtype=torch.int64, device=self.device)
        meta_i32 = torch.empty(2 * b + 1, dtype=torch.int32, device=self.device)
        context_lens, qsl = meta_i32[:b], meta_i32[b:]
        paged_ops.prepare_decode(tables_dev, pos_dev, self.block_size, slot_mapping, context_lens, qsl)
        lens_host = torch.from_numpy(pos + 1)
        metadata = paged_ops.get_scheduler_metadata(
            num_reqs=b, num_heads=self.num_heads, num_kv_heads=self.num_heads, head_dim=self.head_dim,
            seq_lens=lens_host, dtype=self.dtype, query_start_loc=None, causal=False, isa=self.isa,
            block_size=self.block_size)
        return DecodeStep(pos_dev, slot_mapping, context_lens, tables_dev, qsl, metadata, lens_host)

    def stage_cross(self, decoder_layers, request_ids):
        """Cross-attention staging for this batch, rebuilt only when its request ids change."""
        key = tuple(request_ids)
        if key != self._cross_key:
            pages, enc_lens = zip(*(self.cross.pages[rid] for rid in key))
            self._cross_staged = attention.stage_cross(decoder_layers, list(pages), list(enc_lens),
                                                       self.block_size, self.isa)
            self._cross_key = key
        return self._cross_staged
