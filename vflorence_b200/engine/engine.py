"""Continuous-batching decode engine on the paged path (one GPU).

One step (the same order as the reference engine, vflorence/engine/llm_engine.py:57-63):
  1. admit waiting requests while their beams fit in ``max_num_seqs``;
  2. make room for every running row's next token (native runtime; copy-on-write pairs);
  3. encode the step's new requests (one padded batch per image shape) and page their
     encoder K/V into the cross pool, once per request (bf16: projection and page write in one
     tensor-core launch per layer);
  4. copy-on-write copies (one launch, issued before the host packs the rows), device-side step
     metadata (one upload, one kernel), cross staging (memoised on the batch's request ids), then
     one decoder forward;
  5. greedy argmax or beam candidates on the GPU, one small copy back, and the step's
     decisions (forks, finishes, frees) in the native runtime.

The per-row bookkeeping - block tables, reference counts, hypotheses, finished beams - lives in
the host decode runtime (``vflorence_b200.runtime``, C++); Python handles whole requests.
"""

from __future__ import annotations

import contextlib
import math
from collections import deque
from dataclasses import dataclass

import numpy as np
import torch

from .. import paged_ops
from ..block_manager import BlockManager
from ..context import set_context
from ..kv_cache import PagedKVCache
from ..runtime import DecodeRules, DecodeRuntime, StepResult, StepRows
from .model import PagedSeq2Seq
from .sampling import LogitsRules, SamplingParams


@dataclass
class Request:
    input_ids: list[int]
    pixel_values: torch.Tensor | None = None


@dataclass(eq=False)
class _Req:
    """A request's host-side state; its hypotheses live in the native runtime, their decoder
    tokens in rows of the engine's device token buffer."""

    request_id: int
    encoder_ids: list[int]
    params: SamplingParams
    pixel_values: torch.Tensor | None = None


class Engine:
    def __init__(self, hf_model, *, max_num_seqs: int, max_decoder_len: int, max_encoder_len: int,
                 block_size: int = 16, num_blocks: int | None = None, decoder_start_token_id: int | None = None,
                 record_steps: bool = False, cuda_graphs: bool = False, group_beams: bool | str = True,
                 fused_encoder_kv: bool = True, fused_layernorm: bool = True, skinny_linear: bool = True):
        # decoder post-norm residuals: LayerNorm(h + x) in one launch each where it is built for
        # the width (False: the add, then the torch module)
        # float32 steps of at most 16 rows: linear layers as weight-streaming launches (False: GEMMs)
        self.model = PagedSeq2Seq(hf_model, fused_layernorm=fused_layernorm, skinny_linear=skinny_linear)
        # encoder K/V: one tensor-core launch per layer that projects and writes the pages (bf16);
        # False (or another dtype) runs the projection GEMM, then the append kernel
        self.fused_encoder_kv = fused_encoder_kv and paged_ops.kv_proj_supported(
            self.model.dtype, self.model.d_model, self.model.num_heads, self.model.head_dim)
        # beam search: one attention group per request with per-row block tables (bf16, head_dim
        # 64) where enough requests keep the GPU busy ("always": whatever the batch); False
        # attends row by row (the same results, for comparisons)
        self.group_beams = group_beams
        m = self.model
        self.device, self.dtype = m.device, m.dtype
        self.block_size = block_size
        self.max_num_seqs = max_num_seqs
        self.max_decoder_len = max_decoder_len
        self.max_encoder_len = max_encoder_len
        self.num_blocks = num_blocks or max_num_seqs * math.ceil(max_decoder_len / block_size)
        # a row caches at most max_decoder_len tokens: its table never exceeds this
        self.max_blocks = math.ceil((max_decoder_len + 1) / block_size)
        num_cross = max_num_seqs * math.ceil(max_encoder_len / block_size)
        self.kv = PagedKVCache(num_layers=len(m.layers), num_heads=m.num_heads, head_dim=m.head_dim,
                               block_size=block_size, num_blocks=self.num_blocks, num_cross_blocks=num_cross,
                               dtype=self.dtype, device=self.device)
        self.kv.bind(m.layers)
        cfg = hf_model.config.get_text_config()
        self.start_token = cfg.decoder_start_token_id if decoder_start_token_id is None else decoder_start_token_id
        self._make_runtime(4)
        M, W = max_num_seqs, self.max_blocks
        self._eager_host = torch.zeros(M * (W + 1), dtype=torch.int32).pin_memory()
        self._meta_host = torch.zeros(5 * M, dtype=torch.int32).pin_memory()
        self._meta_dev = torch.zeros(5 * M, dtype=torch.int32, device=self.device)
        self._born_host = self._born_dev = None
        self.waiting: deque[_Req] = deque()
        self.requests: dict[int, _Req] = {}  # admitted and not finished
        self.outputs: dict[int, list[int]] = {}
        self._next_id = 0
        self._rules: tuple[SamplingParams, LogitsRules, DecodeRules] | None = None
        self.record = [] if record_steps else None
        # a PhaseTimer (engine.timing) to bracket the job's phases with CUDA events, or None
        self.timer = None
        self.graphs = None
        if cuda_graphs:
            from .graphs import GraphedDecoder

            self.graphs = GraphedDecoder(self)

    def _make_runtime(self, slots_per_row: int) -> None:
        """Hypothesis slots (token rows) for ``slots_per_row`` per running row: a beam step holds
        the parents, up to beams_to_keep children per request and the kept finished beams."""
        self.slots_per_row = slots_per_row
        self.num_slots = slots_per_row * self.max_num_seqs + 4
        self.rt = DecodeRuntime(self.num_blocks, self.block_size, self.num_slots, self.max_blocks)
        self.blocks = BlockManager.over(self.rt)
        self.tokens = torch.zeros(self.num_slots, self.max_decoder_len + 2, dtype=torch.int32, device=self.device)

    # -------------------------------------------------------------------------------- requests
    def add_request(self, request: Request, params: SamplingParams) -> int:
        vocab = self.model.lm.get_input_embeddings().num_embeddings
        if any(not 0 <= t < vocab for t in request.input_ids):
            raise ValueError(f"encoder prompt holds token ids outside [0, {vocab})")
        if len(request.input_ids) > self.max_encoder_len:
            raise ValueError(f"encoder prompt has {len(request.input_ids)} tokens (max {self.max_encoder_len})")
        if params.max_tokens > self.max_decoder_len:
            raise ValueError(f"max_tokens {params.max_tokens} exceeds max_decoder_len {self.max_decoder_len}")
        if params.num_beams > self.max_num_seqs:
            raise ValueError("num_beams exceeds max_num_seqs")
        if params.beams_to_keep() > paged_ops.MAX_TOPK:
            raise ValueError(f"beam search keeps {params.beams_to_keep()} candidates per row; the device "
                             f"selection is built for at most {paged_ops.MAX_TOPK}")
        if self.waiting or self.requests:
            other = (self.waiting[0] if self.waiting else next(iter(self.requests.values()))).params
            if other != params:
                raise ValueError("all active requests must share the same SamplingParams")
        else:
            need = 2 + params.beams_to_keep() // params.num_beams if params.num_beams > 1 else 1
            if need > self.slots_per_row:
                self._make_runtime(need)
        rid = self._next_id
        self._next_id += 1
        self.waiting.append(_Req(rid, list(request.input_ids), params, request.pixel_values))
        return rid

    def is_finished(self) -> bool:
        return not self.waiting and not self.requests

    @torch.inference_mode()
    def generate(self, requests, params: SamplingParams) -> list[list[int]]:
        ids = [self.add_request(r, params) for r in requests]
        try:
            while not self.is_finished():
                self.step()
        except BaseException:
            self.abort()
            raise
        return [self.outputs.pop(i) for i in ids]

    def abort(self) -> None:
        self.waiting.clear()
        self.requests.clear()
        self.rt.reset()
        self.kv.reset()
        set_context()

    # ------------------------------------------------------------------------------------ step
    @torch.inference_mode()
    def step(self) -> list[int]:
        """One decode step; returns the ids of the requests it finished."""
        if self.timer is None:
            return self._step()
        with self.timer("step"):
            return self._step()

    def _phase(self, name: str):
        return self.timer(name) if self.timer is not None else contextlib.nullcontext()

    def _step(self) -> list[int]:
        params = self._admit()
        n = self.rt.num_running
        if n == 0:
            return []
        copies = self.rt.prepare_step()
        # copy-on-write first: the GPU copies the blocks while the host packs the step's rows
        # (the copies touch only the self pools; nothing below reads or writes those blocks first)
        self.kv.copy_blocks(copies, checked=True)
        g = self.graphs.graph_for(n, params.num_beams) if self.graphs is not None else None
        if g is not None:
            rows = self.rt.pack_step(*g.host_views())
        else:
            W = self.max_blocks
            host = self._eager_host.numpy()[: n * W + n]
            rows = self.rt.pack_step(host[: n * W].reshape(n, W), host[n * W:])
        fresh = np.flatnonzero(rows.positions == 0)
        if len(fresh):
            self._encode([self.requests[int(r)] for r in rows.request_ids[fresh]])
        if self.record is not None:
            tables = g.host_views()[0] if g is not None else host[: n * W].reshape(n, W)
            self.record.append({"request_ids": rows.request_ids.tolist(), "positions": rows.positions.tolist(),
                                "block_tables": [tables[i, :k].tolist() for i, k in enumerate(rows.table_lens)],
                                "copies": [tuple(c) for c in copies.tolist()]})
        if g is not None:
            logits = g.launch(rows)
        else:
            st = self.kv.prepare_decode_host(self._eager_host[: n * W + n], n, W)
            staged = self.kv.stage_cross(self.model.layers, rows.request_ids.tolist())
            self_kw = dict(self_metadata=st.self_metadata)
            if (params.num_beams > 1 and self.group_beams and paged_ops.row_tables_supported(self.dtype,
                                                                                           self.model.head_dim)
                    and (self.group_beams == "always"
                         or paged_ops.row_tables_pay_off(rows.num_groups, self.model.num_heads))):
                self_kw = self._beam_groups(rows)
            set_context(context_lens=st.context_lens, block_tables=st.block_tables, slot_mapping=st.slot_mapping,
                        query_start_loc=st.query_start_loc, isa=self.kv.isa, cross_staged=staged, **self_kw)
            try:
                ids = torch.from_numpy(rows.tokens).to(self.device, non_blocking=True)
                logits = self.model.decode(ids.long(), st.positions.long())
            finally:
                set_context()
        meta = self._upload_rows(rows)
        if params.num_beams == 1:
            return self._finish_greedy(params, rows, meta, logits)
        return self._finish_beam(params, rows, meta, logits)

    def _admit(self) -> SamplingParams | None:
        """Admit waiting requests while their beams fit (scheduler.py:37-48)."""
        used = sum(r.params.num_beams for r in self.requests.values())
        admitted = []
        while self.waiting and used + self.waiting[0].params.num_beams <= self.max_num_seqs:
            r = self.waiting.popleft()
            admitted.append(self.rt.admit(r.request_id, self.start_token))
            self.requests[r.request_id] = r
            used += r.params.num_beams
        if admitted:
            self.tokens[torch.tensor(admitted, device=self.device), 0] = self.start_token
        return next(iter(self.requests.values())).params if self.requests else None

    def _encode(self, fresh) -> None:
        """Page the encoder K/V of this step's new requests.

        Encoder pages are assigned as the reference does (groups of equal prompt length and
        image shape, in order of first appearance, vflorence/engine/model_runner.py:215-242).
        The encoder itself runs once per image shape: shorter prompts are right-padded with an
        attention mask, and padded positions get slot -1, so one append per layer writes only
        real tokens.
        """
        bs = self.block_size
        groups: dict = {}
        for s in fresh:
            key = (len(s.encoder_ids), None if s.pixel_values is None else tuple(s.pixel_values.shape))
            groups.setdefault(key, []).append(s)
        for (enc_len, _), group in groups.items():
            self.kv.cross.assign([s.request_id for s in group], enc_len, bs)
        batches: dict = {}
        for s in fresh:
            batches.setdefault(None if s.pixel_values is None else tuple(s.pixel_values.shape), []).append(s)
        pad_id = self.model.lm.config.pad_token_id or 0
        for px, batch in batches.items():
            width = max(len(s.encoder_ids) for s in batch)
            ids = torch.full((len(batch), width), pad_id, dtype=torch.long)
            mask = torch.zeros((len(batch), width), dtype=torch.long)
            slots = torch.full((len(batch), width), -1, dtype=torch.long)
            for i, s in enumerate(batch):
                n = len(s.encoder_ids)
                ids[i, :n] = torch.tensor(s.encoder_ids)
                mask[i, :n] = 1
                pages = self.kv.cross.pages[s.request_id][0].long()
                t = torch.arange(n)
                slots[i, :n] = pages[t // bs] * bs + t % bs
            ragged = bool((mask == 0).any())
            # pinned staging: the uploads queue on the stream without waiting for it
            up = lambda t: t.pin_memory().to(self.device, non_blocking=True)  # noqa: E731
            ids, slots = up(ids), up(slots.view(-1))
            pix = None
            if px is not None:  # one copy per image into the batch (asynchronous from pinned memory)
                pix = torch.empty((len(batch),) + px, dtype=batch[0].pixel_values.dtype, device=self.device)
                for i, s in enumerate(batch):
                    pix[i].copy_(s.pixel_values, non_blocking=True)
            hidden = self.model.encode(ids, pix, up(mask) if ragged else None, phase=self._phase)
            with self._phase("encoder_kv_pages"):
                for layer in range(len(self.model.layers)):
                    if self.fused_encoder_kv:
                        L = self.model.layers[layer]
                        self.kv.project_encoder_kv(layer, hidden.reshape(-1, self.model.d_model), L.w_kv, L.b_kv,
                                                   slots)
                    else:
                        k, v = self.model.cross_kv(layer, hidden)
                        self.kv.write_encoder_kv(layer, k, v, slots)

    def _beam_groups(self, rows: StepRows) -> dict:
        """Self-attention groups of an eager beam step: runs of consecutive rows of one request
        (the same position), a row-tables plan, one upload of the groups' offsets and lengths."""
        rid = rows.request_ids
        starts = np.flatnonzero(np.r_[True, rid[1:] != rid[:-1]])
        qsl = np.r_[starts, rows.n].astype(np.int32)
        lens = (rows.positions[starts] + 1).astype(np.int32)
        m = self.model
        meta = paged_ops.get_scheduler_metadata(len(starts), m.num_heads, m.num_heads, m.head_dim,
                                                torch.from_numpy(lens), self.dtype, torch.from_numpy(qsl), False,
                                                self.kv.isa, self.block_size, row_tables=True)
        dev = torch.from_numpy(np.r_[qsl, lens]).to(self.device)
        return dict(self_metadata=meta, self_groups=dev[: len(qsl)], self_group_lens=dev[len(qsl):])

    def _rules_for(self, params: SamplingParams) -> tuple[LogitsRules, DecodeRules]:
        if self._rules is None or self._rules[0] is not params:
            self._rules = (params, LogitsRules(params, self.model.vocab_size, self.device),
                           DecodeRules.from_params(params))
        return self._rules[1], self._rules[2]

    def _upload_rows(self, rows: StepRows) -> torch.Tensor:
        """Rows' slots, lengths, request groups, ranks and cumulative log-probs on the device:
        int32 [5, n] (the last row holds float32 bits), one pinned copy."""
        n = rows.n
        host = self._meta_host.numpy()[: 5 * n].reshape(5, n)
        host[0], host[1], host[2], host[3] = rows.slots, rows.lengths, rows.groups, rows.ranks
        host[4] = rows.cum_logprobs.view(np.int32)
        dev = self._meta_dev[: 5 * n]
        dev.copy_(self._meta_host[: 5 * n], non_blocking=True)
        return dev.view(5, n)

    def _emit(self, res: StepResult) -> list[int]:
        """Record finished requests' generated tokens (one copy for the step) and release them."""
        done = res.done_request.tolist()
        if not done:
            return done
        width = int(res.done_length.max())
        slots = torch.from_numpy(res.done_slot.astype(np.int64)).to(self.device)
        rows = self.tokens[slots, :width].cpu().numpy()
        for rid, row, length in zip(done, rows, res.done_length.tolist()):
            self.outputs[rid] = row[1:length].tolist()
            self.kv.clear_request(rid)
            del self.requests[rid]
        return done

    def _finish_greedy(self, params, rows: StepRows, meta: torch.Tensor, logits) -> list[int]:
        rules, drules = self._rules_for(params)
        slots, lengths = meta[0].long(), meta[1].long()
        scores = logits
        if rules.active:
            hist = self.tokens[slots] if rules.needs_history else None
            scores = rules(logits.float(), hist, lengths)
        _, picks = paged_ops.row_topk(scores, 1)  # the argmax, first index on ties
        picks = picks.view(-1)
        self.tokens[slots, lengths] = picks
        res = self.rt.advance_greedy(drules, picks.cpu().numpy())
        return self._emit(res)

    def _beam_candidates(self, rows: StepRows, meta: torch.Tensor, logits: torch.Tensor, scores, keep: int) -> np.ndarray:
        """Each request's best ``keep`` (row, token, cum_logprob) continuations, selected on the
        GPU: every row's top-k log-probs plus its cumulative log-prob (one fused kernel over the
        logits, or over the rule-processed scores), then one merge per request in the order of
        a stable descending sort of its rows' lists - the reference's stable Python sort of the
        concatenated rows (vflorence/engine/model_runner.py:383-410).
        Returns int32 [3, requests, keep] (row, token, float32 bits of the score); row -1 = none."""
        vocab = logits.shape[1]
        k = min(keep, vocab)
        cum = meta[4].view(torch.float32)
        if scores is None:
            values, ids = paged_ops.row_topk(logits, k, log_softmax=True, row_offset=cum)
        else:
            values, ids = paged_ops.row_topk(scores, k, row_offset=cum)
        return paged_ops.beam_merge(values, ids, meta[2], meta[3], rows.num_groups, keep).cpu().numpy()

    def _finish_beam(self, params, rows: StepRows, meta: torch.Tensor, logits) -> list[int]:
        rules, drules = self._rules_for(params)
        scores = None
        if rules.active:
            hist = self.tokens[meta[0].long()] if rules.needs_history else None
            scores = rules(torch.log_softmax(logits.float(), dim=-1), hist, meta[1].long())
        cand = self._beam_candidates(rows, meta, logits, scores, params.beams_to_keep())
        res = self.rt.advance_beam(drules, cand[0], cand[1], cand[2].view(np.float32))
        nb = len(res.born_child)
        if nb:  # children's token rows: the parent's row plus the new token
            if self._born_host is None or self._born_host.numel() < 4 * nb:
                self._born_host = torch.zeros(max(4 * nb, 4096), dtype=torch.int32).pin_memory()
                self._born_dev = torch.zeros_like(self._born_host, device=self.device)
            host = self._born_host.numpy()[: 4 * nb].reshape(4, nb)
            host[0], host[1], host[2], host[3] = res.born_parent, res.born_child, res.born_pos, res.born_token
            dev = self._born_dev[: 4 * nb]
            dev.copy_(self._born_host[: 4 * nb], non_blocking=True)
            paged_ops.fork_token_rows(self.tokens, dev.view(4, nb))
        return self._emit(res)
