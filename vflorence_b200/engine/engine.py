"""Continuous-batching decode engine on the paged path (one GPU).

One step (the same order as the reference engine, vflorence/engine/llm_engine.py:57-63):
  1. admit waiting requests while their beams fit in ``max_num_seqs``;
  2. make room for every running sequence's next token (BlockManager; copy-on-write pairs);
  3. encode the step's new requests (grouped by prompt length and image shape) and page their
     encoder K/V into the cross pool, once per request;
  4. copy-on-write copies (one launch), device-side step metadata (one upload, one kernel),
     cross staging (memoised on the batch's request ids), then one decoder forward;
  5. greedy argmax or beam candidates on the GPU; forks, finishes and frees on the host.
"""

from __future__ import annotations

import math
from collections import deque
from dataclasses import dataclass, field

import torch

from ..block_manager import BlockManager
from ..context import set_context
from ..kv_cache import PagedKVCache
from .model import PagedSeq2Seq
from .sampling import LogitsRules, SamplingParams


@dataclass
class Request:
    input_ids: list[int]
    pixel_values: torch.Tensor | None = None


@dataclass(eq=False)
class _Seq:
    """One hypothesis. Its decoder tokens live in row ``slot`` of the engine's device token
    buffer (start token first); the host keeps only the last token and the length."""

    request_id: int
    encoder_ids: list[int]
    params: SamplingParams
    slot: int
    last_token: int
    length: int = 1
    pixel_values: torch.Tensor | None = None
    block_table: list[int] = field(default_factory=list)
    num_cached_tokens: int = 0
    cum_logprob: float = 0.0
    prompt_len: int = 1

    @property
    def num_generated(self) -> int:
        return self.length - self.prompt_len

    def finished(self, eos: set[int]) -> bool:
        return self.last_token in eos or self.num_generated >= self.params.max_tokens

    def score(self) -> float:
        return self.cum_logprob / (max(self.num_generated, 1) ** self.params.length_penalty)


class Engine:
    def __init__(self, hf_model, *, max_num_seqs: int, max_decoder_len: int, max_encoder_len: int,
                 block_size: int = 16, num_blocks: int | None = None, decoder_start_token_id: int | None = None,
                 record_steps: bool = False, cuda_graphs: bool = False):
        self.model = PagedSeq2Seq(hf_model)
        m = self.model
        self.device, self.dtype = m.device, m.dtype
        self.block_size = block_size
        self.max_num_seqs = max_num_seqs
        self.max_decoder_len = max_decoder_len
        self.max_encoder_len = max_encoder_len
        self.num_blocks = num_blocks or max_num_seqs * math.ceil(max_decoder_len / block_size)
        num_cross = max_num_seqs * math.ceil(max_encoder_len / block_size)
        self.kv = PagedKVCache(num_layers=len(m.layers), num_heads=m.num_heads, head_dim=m.head_dim,
                               block_size=block_size, num_blocks=self.num_blocks, num_cross_blocks=num_cross,
                               dtype=self.dtype, device=self.device)
        self.kv.bind(m.layers)
        self.blocks = BlockManager(self.num_blocks, block_size)
        cfg = hf_model.config.get_text_config()
        self.start_token = cfg.decoder_start_token_id if decoder_start_token_id is None else decoder_start_token_id
        # decoder tokens of every live hypothesis, one row each. Beam children take fresh rows,
        # so a step can hold parents, their children (up to 2 per kept beam) and the finished
        # hypotheses kept per request: at most 4 rows per sequence slot
        self.tokens = torch.zeros(4 * max_num_seqs + 4, max_decoder_len + 2, dtype=torch.int32, device=self.device)
        self.free_slots = list(range(self.tokens.shape[0]))
        self.waiting: deque[_Seq] = deque()
        self.running: list[_Seq] = []
        self.finished_beams: dict[int, list[_Seq]] = {}
        self.outputs: dict[int, list[int]] = {}
        self._next_id = 0
        self._rules: tuple[SamplingParams, LogitsRules] | None = None
        self.record = [] if record_steps else None
        self.graphs = None
        if cuda_graphs:
            from .graphs import GraphedDecoder

            self.graphs = GraphedDecoder(self)

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
        if self.waiting or self.running:
            other = (self.waiting or self.running)[0].params
            if other != params:
                raise ValueError("all active requests must share the same SamplingParams")
        rid = self._next_id
        self._next_id += 1
        self.waiting.append(_Seq(rid, list(request.input_ids), params, -1, self.start_token,
                                 pixel_values=request.pixel_values))
        return rid

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

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
        self.running.clear()
        self.finished_beams.clear()
        self.blocks.reset()
        self.kv.reset()
        self.free_slots = list(range(self.tokens.shape[0]))
        set_context()

    # ------------------------------------------------------------------------------------ step
    @torch.inference_mode()
    def step(self) -> list[int]:
        seqs, copies = self._schedule()
        if not seqs:
            return []
        fresh = [s for s in seqs if s.num_cached_tokens == 0]
        if fresh:
            self._encode(fresh)
        self.kv.copy_blocks(copies)
        tables = [s.block_table for s in seqs]
        positions = [s.num_cached_tokens for s in seqs]
        if self.record is not None:
            self.record.append({"request_ids": [s.request_id for s in seqs], "positions": list(positions),
                                "block_tables": [list(t) for t in tables], "copies": list(copies)})
        logits = self.graphs.run(seqs) if self.graphs is not None else None
        if logits is None:  # eager step
            st = self.kv.prepare_decode(tables, positions)
            staged = self.kv.stage_cross(self.model.layers, [s.request_id for s in seqs])
            set_context(context_lens=st.context_lens, block_tables=st.block_tables, slot_mapping=st.slot_mapping,
                        query_start_loc=st.query_start_loc, self_metadata=st.self_metadata, isa=self.kv.isa,
                        cross_staged=staged)
            try:
                ids = torch.tensor([s.last_token for s in seqs], dtype=torch.long).pin_memory()
                logits = self.model.decode(ids.to(self.device, non_blocking=True), st.positions.long())
            finally:
                set_context()
        for s in seqs:
            s.num_cached_tokens += 1
        if seqs[0].params.num_beams == 1:
            return self._finish_greedy(seqs, logits)
        return self._finish_beam(seqs, logits)

    def _schedule(self):
        used = sum({s.request_id: s.params.num_beams for s in self.running}.values())
        admitted = []
        while self.waiting and used + self.waiting[0].params.num_beams <= self.max_num_seqs:
            s = self.waiting.popleft()
            s.slot = self.free_slots.pop()
            self.running.append(s)
            admitted.append(s.slot)
            used += s.params.num_beams
        if admitted:
            self.tokens[torch.tensor(admitted, device=self.device), 0] = self.start_token
        seqs = list(self.running)
        if self.blocks.required_new_blocks(seqs) > self.blocks.num_free_blocks:
            raise RuntimeError("KV cache is full; increase num_blocks")
        copies = [c for s in seqs if (c := self.blocks.ensure_capacity(s)) is not None]
        return seqs, copies

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
            ids, slots = ids.to(self.device), slots.view(-1).to(self.device)
            pix = None if px is None else torch.stack([s.pixel_values for s in batch]).to(self.device)
            hidden = self.model.encode(ids, pix, mask.to(self.device) if ragged else None)
            for layer in range(len(self.model.layers)):
                k, v = self.model.cross_kv(layer, hidden)
                self.kv.write_encoder_kv(layer, k, v, slots)

    def _rules_for(self, params: SamplingParams) -> LogitsRules:
        if self._rules is None or self._rules[0] is not params:
            self._rules = (params, LogitsRules(params, self.model.vocab_size, self.device))
        return self._rules[1]

    def _rows_state(self, seqs):
        """Device views for the rules: token rows and lengths of ``seqs``."""
        meta = torch.tensor([[s.slot for s in seqs], [s.length for s in seqs]], dtype=torch.long).pin_memory()
        meta = meta.to(self.device, non_blocking=True)
        rules = self._rules_for(seqs[0].params)
        hist = self.tokens[meta[0]] if rules.needs_history else None
        return rules, meta[0], meta[1], hist

    def _emit(self, done: list[_Seq]) -> None:
        """Record finished hypotheses' generated tokens (one copy for the step) and release them."""
        if not done:
            return
        width = max(s.length for s in done)
        rows = self.tokens[torch.tensor([s.slot for s in done], device=self.device), :width].tolist()
        for s, row in zip(done, rows):
            self.outputs[s.request_id] = row[s.prompt_len: s.length]
            self.kv.clear_request(s.request_id)

    def _remove(self, seq: _Seq) -> None:
        self.running.remove(seq)
        self.blocks.deallocate(seq)
        self.free_slots.append(seq.slot)

    def _finish_greedy(self, seqs, logits) -> list[int]:
        params = seqs[0].params
        rules, slots, lengths, hist = self._rows_state(seqs)
        picks = rules(logits.float(), hist, lengths).argmax(dim=-1)
        self.tokens[slots, lengths] = picks.to(torch.int32)
        eos = set(params.eos_ids())
        done = []
        for s, t in zip(seqs, picks.tolist()):
            s.last_token, s.length = t, s.length + 1
            if s.finished(eos):
                done.append(s)
        self._emit(done)
        for s in done:
            self._remove(s)
        return [s.request_id for s in done]

    def _beam_candidates(self, seqs, scores, keep):
        """Each request's best ``keep`` (row, token, cum_logprob) continuations, selected on the
        GPU: every row's top-k plus its cumulative log-prob, scattered into a per-request grid in
        row order, one stable descending sort per request - the order the reference's stable
        Python sort of the concatenated rows gives (vflorence/engine/model_runner.py:383-410)."""
        rows, vocab = scores.shape
        k = min(keep, vocab)
        req_of, slot_of, counts, order = [], [], [], {}
        for s in seqs:
            r = order.get(s.request_id)
            if r is None:
                r = order[s.request_id] = len(counts)
                counts.append(0)
            req_of.append(r)
            slot_of.append(counts[r])
            counts[r] += 1
        R, width = len(counts), max(counts)
        host = torch.tensor([req_of, slot_of], dtype=torch.long).pin_memory()
        cum = torch.tensor([s.cum_logprob for s in seqs], dtype=torch.float32).pin_memory()
        idx = host.to(self.device, non_blocking=True)
        top_s, top_i = torch.topk(scores, k, dim=-1)
        top_s += cum.to(self.device, non_blocking=True).unsqueeze(-1)
        grid_s = torch.full((R, width, k), float("-inf"), device=self.device)
        grid_t = torch.zeros((R, width, k), dtype=torch.long, device=self.device)
        grid_r = torch.full((R, width, k), -1, dtype=torch.long, device=self.device)
        grid_s[idx[0], idx[1]] = top_s
        grid_t[idx[0], idx[1]] = top_i
        grid_r[idx[0], idx[1]] = torch.arange(rows, device=self.device).unsqueeze(-1).expand(rows, k)
        srt, pos = torch.sort(grid_s.view(R, width * k), dim=1, descending=True, stable=True)
        n = min(keep, width * k)
        pos = pos[:, :n]
        picked = torch.stack([grid_r.view(R, -1).gather(1, pos).double(), grid_t.view(R, -1).gather(1, pos).double(),
                              srt[:, :n].double()]).tolist()
        rids = list(order)
        cands = {}
        for r in range(R):
            cands[rids[r]] = [(int(row), int(tok), sc) for row, tok, sc in zip(*(picked[c][r] for c in range(3)))
                              if row >= 0]
        return cands

    def _child(self, parent: _Seq, token: int, cum_logprob: float) -> _Seq:
        return _Seq(parent.request_id, parent.encoder_ids, parent.params, self.free_slots.pop(), token,
                    parent.length + 1, parent.pixel_values, [], parent.num_cached_tokens, cum_logprob,
                    parent.prompt_len)

    def _finish_beam(self, seqs, logits) -> list[int]:
        params = seqs[0].params
        rules, slots, lengths, hist = self._rows_state(seqs)
        scores = rules(torch.log_softmax(logits.float(), dim=-1), hist, lengths)
        cands = self._beam_candidates(seqs, scores, params.beams_to_keep())
        eos = set(params.eos_ids())
        nb = params.num_beams
        born = []   # (parent, child): every child whose tokens must be written this step
        done_rids, emitted, released = [], [], []
        for rid, cand in cands.items():
            finished = self.finished_beams.setdefault(rid, [])
            running = []
            for rank, (row, token, cum) in enumerate(cand):
                if rank >= nb and len(running) >= nb:
                    break
                parent = seqs[row]
                is_done = token in eos or parent.num_generated + 1 >= params.max_tokens
                if is_done and rank >= nb:
                    continue
                if not is_done and len(running) >= nb:
                    continue
                child = self._child(parent, token, cum)
                born.append((parent, child))
                (finished if is_done else running).append(child if is_done else (parent, child))
            finished.sort(key=lambda c: c.score(), reverse=True)
            for dropped in finished[nb:]:
                released.append(dropped)
            del finished[nb:]
            best_running = max((c.score() for _, c in running), default=float("-inf"))
            stop = len(finished) >= nb and (params.early_stopping or finished[-1].score() >= best_running)
            if not running or stop:
                self.finished_beams.pop(rid, None)
                emitted.append(finished[0])
                released.extend(finished)
                released.extend(c for _, c in running)
                done_rids.append(rid)
            else:
                for parent, child in running:
                    self.blocks.fork(parent, child)
                    self.running.append(child)
        if born:  # children's token rows: the parent's row plus the new token
            meta = torch.tensor([[p.slot for p, _ in born], [c.slot for _, c in born],
                                 [p.length for p, _ in born], [c.last_token for _, c in born]],
                                dtype=torch.long).pin_memory().to(self.device, non_blocking=True)
            self.tokens[meta[1]] = self.tokens[meta[0]]
            self.tokens[meta[1], meta[2]] = meta[3].to(torch.int32)
        self._emit(emitted)
        for s in seqs:
            self._remove(s)
        for c in released:  # finished hypotheses hold a token row but no blocks
            self.free_slots.append(c.slot)
        return done_rids
