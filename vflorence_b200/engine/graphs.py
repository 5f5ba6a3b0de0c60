"""CUDA-graph replay of the decoder step (one graph per padded batch size).

A decode step launches a few hundred kernels (GEMMs, norms, the paged ops); launched one by one
from Python the step is bound by the host. Here each batch-size bucket captures, once, the
device-side step metadata kernel plus the whole decoder forward into a CUDA graph over static
buffers; a step then is one pinned upload of its block tables, positions and token ids, and one
replay.

What makes a captured step valid for any batch of up to B rows:
  * rows past the real batch are padding: position -1, so the metadata kernel gives them slot -1
    (no append) and context length 0 (zero attention output); their logits are ignored;
  * the attention plans are made for the worst case (every row at max_decoder_len, every
    request at max_encoder_len, ``beams`` rows per request), so the captured grids cover any real
    batch; CTAs beyond a row's real length exit at once;
  * cross-attention staging (pages, lengths, beam grouping) lives in static buffers refreshed
    only when the batch's request ids change.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from .. import paged_ops
from ..attention import group_rows
from ..context import get_context, set_context

BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 384, 448, 512)


class _StepGraph:
    def __init__(self, engine, rows: int, beams: int, pool):
        e = engine
        m, kv = e.model, e.kv
        self.e, self.rows, self.beams = e, rows, beams
        bs = e.block_size
        self.width = math.ceil(e.max_decoder_len / bs)
        self.cwidth = math.ceil(e.max_encoder_len / bs)
        dev = e.device
        B, M, Mc = rows, self.width, self.cwidth
        # per-step inputs: tables [B, M] | positions [B] | token ids [B]
        self.host_in = torch.zeros(B * M + 2 * B, dtype=torch.int32).pin_memory()
        self.dev_in = torch.zeros_like(self.host_in, device=dev)
        self.tables = self.dev_in[: B * M].view(B, M)
        self.pos = self.dev_in[B * M: B * M + B]
        self.ids = self.dev_in[B * M + B:]
        self.slots = torch.full((B,), -1, dtype=torch.int64, device=dev)
        meta = torch.zeros(2 * B + 1, dtype=torch.int32, device=dev)
        self.ctx_lens, self.qsl = meta[:B], meta[B:]
        # cross staging: tables [B, Mc] | lengths [B] | query_start_loc [B + 1]
        self.host_cross = torch.zeros(B * Mc + 2 * B + 1, dtype=torch.int32).pin_memory()
        self.dev_cross = torch.zeros_like(self.host_cross, device=dev)
        self.ctab = self.dev_cross[: B * Mc].view(B, Mc)
        self.clens = self.dev_cross[B * Mc: B * Mc + B]
        self.cqsl = self.dev_cross[B * Mc + B:]
        self.cross_key = None
        self.copy_done = torch.cuda.Event()
        H, D = m.num_heads, m.head_dim
        plan_qsl = torch.tensor([min(r * beams, B) for r in range(B + 1)], dtype=torch.int32)
        # beam search: the beams of a request (the cross-staging groups) attend as one group with
        # per-row block tables; the groups' lengths are gathered from the rows' in the graph
        self.grouped = (beams > 1 and e.group_beams and paged_ops.row_tables_supported(e.dtype, D)
                        and (e.group_beams == "always" or paged_ops.row_tables_pay_off(math.ceil(B / beams), H)))
        self.meta_self = paged_ops.get_scheduler_metadata(
            B, H, H, D, torch.full((B,), e.max_decoder_len, dtype=torch.int32), e.dtype,
            plan_qsl if self.grouped else None, False, kv.isa, bs, row_tables=self.grouped)
        self.meta_cross = paged_ops.get_scheduler_metadata(
            B, H, H, D, torch.full((B,), e.max_encoder_len, dtype=torch.int32), e.dtype, plan_qsl, False,
            kv.isa, bs)
        self.staged = [(kv.cross_k_caches[i], kv.cross_v_caches[i], self.ctab, self.clens, self.meta_cross, self.cqsl)
                       for i in range(len(m.layers))]
        # padding everywhere, then warm up and capture
        hv = self.host_in.numpy()
        hv[B * M: B * M + B] = -1
        self.dev_in.copy_(self.host_in)
        self.dev_cross.zero_()
        self._set_context()
        try:
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                for _ in range(2):
                    self._forward()
            torch.cuda.current_stream(dev).wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, pool=pool):
                self.logits = self._forward()
        finally:
            set_context()

    def _set_context(self):
        set_context(context_lens=self.ctx_lens, block_tables=self.tables, slot_mapping=self.slots,
                    query_start_loc=self.qsl, self_metadata=self.meta_self, isa=self.e.kv.isa,
                    cross_staged=self.staged)

    def _forward(self):
        paged_ops.prepare_decode(self.tables, self.pos, self.e.block_size, self.slots, self.ctx_lens, self.qsl)
        if self.grouped:
            ctx = get_context()
            ctx.self_groups = self.cqsl
            # a group's length is its first row's; groups without rows read any row
            ctx.self_group_lens = self.ctx_lens.index_select(0, self.cqsl[:-1].clamp(max=self.rows - 1))
        return self.e.model.decode(self.ids.long(), self.pos.long())

    def host_views(self):
        """Pinned upload views (tables [B, M], positions [B], token ids [B]) for the runtime to
        pack the step's rows into; waits until the previous upload has left them."""
        self.copy_done.synchronize()
        B, M = self.rows, self.width
        hv = self.host_in.numpy()
        return hv[: B * M].reshape(B, M), hv[B * M: B * M + B], hv[B * M + B:]

    def launch(self, rows) -> torch.Tensor:
        """Replay for the packed rows; rows past ``rows.n`` are padding. Logits [n, vocab]."""
        b, B, M = rows.n, self.rows, self.width
        self.host_in.numpy()[B * M + b: B * M + B] = -1
        self.dev_in.copy_(self.host_in, non_blocking=True)
        if self.cross_key is None or not np.array_equal(self.cross_key, rows.request_ids):
            self._stage_cross(rows.request_ids.tolist())
            self.cross_key = rows.request_ids.copy()
        self.copy_done.record()
        self.graph.replay()
        return self.logits[:b]

    def _stage_cross(self, request_ids):
        B, Mc = self.rows, self.cwidth
        pages, lens = zip(*(self.e.kv.cross.pages[r] for r in request_ids))
        firsts, offsets = group_rows(list(pages), list(lens))
        hc = self.host_cross.numpy()
        ctab = hc[: B * Mc].reshape(B, Mc)
        ctab[:] = 0
        clens = hc[B * Mc: B * Mc + B]
        clens[:] = 0
        cqsl = hc[B * Mc + B:]
        cqsl[:] = len(request_ids)
        for g, i in enumerate(firsts):
            ctab[g, : pages[i].numel()] = pages[i].numpy()
            clens[g] = lens[i]
        cqsl[: len(offsets)] = offsets
        self.dev_cross.copy_(self.host_cross, non_blocking=True)


class GraphedDecoder:
    """Captured decoder steps keyed by (padded rows, rows per request)."""

    def __init__(self, engine):
        self.e = engine
        self.graphs: dict[tuple[int, int], _StepGraph] = {}

    @staticmethod
    def bucket(rows: int) -> int | None:
        for b in BUCKETS:
            if b >= rows:
                return b
        return None

    def capture(self, max_rows: int, beams: int) -> None:
        """Capture every bucket up to ``max_rows`` rows ahead of time (start-up cost, not per step)."""
        for rows in BUCKETS:
            if rows > max_rows and rows != self.bucket(max_rows):
                break
            if (rows, beams) not in self.graphs:
                self.graphs[(rows, beams)] = _StepGraph(self.e, rows, beams, None)

    def graph_for(self, rows: int, beams: int) -> _StepGraph | None:
        """The captured step for ``rows`` running rows, or None when the batch is larger than
        every bucket (the step then runs eagerly)."""
        b = self.bucket(rows)
        if b is None:
            return None
        key = (b, beams)
        g = self.graphs.get(key)
        if g is None:
            g = self.graphs[key] = _StepGraph(self.e, b, beams, None)  # own memory pool
        return g
