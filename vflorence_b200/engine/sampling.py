"""Decoding rules of the engine: transformers' logits rules and beam bookkeeping, restated.

The decisions must equal the reference engine's (vflorence/layers/logits_processor.py,
vflorence/engine/model_runner.py:343-410, vflorence/engine/scheduler.py:83-127), which follow
HuggingFace ``generate``:

* rules, in this order: repetition penalty, no-repeat n-gram ban, minimum length (EOS banned
  while the decoder sequence is shorter than ``min_length``), forced BOS at the first generated
  position, forced EOS at the last one, token suppression, begin-suppression at the first
  generated position. Lengths count the decoder start token.
* greedy: argmax of the processed logits.
* beam search: processed log-probs, top ``K = max(2, 1 + #eos) * num_beams`` per row plus the
  row's cumulative log-prob, a request's rows merged and sorted (stable) by score, the best K
  kept. A candidate ending in EOS (or reaching max_tokens) is finished only when its rank is
  below num_beams; at most num_beams continue. Finished hypotheses are ranked by
  ``cum_logprob / max(generated, 1) ** length_penalty``; a request stops when nothing runs, or
  when num_beams hypotheses are finished and either early_stopping is set or the worst kept
  finished score beats the best running one.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

NEG_INF = float("-inf")


@dataclass
class SamplingParams:
    max_tokens: int = 64
    num_beams: int = 1
    repetition_penalty: float = 1.0
    eos_token_id: int | list[int] | None = None
    length_penalty: float = 1.0
    no_repeat_ngram_size: int = 0
    min_length: int = 0
    forced_bos_token_id: int | None = None
    forced_eos_token_id: int | list[int] | None = None
    suppress_tokens: list[int] | None = None
    begin_suppress_tokens: list[int] | None = None
    early_stopping: bool = False
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        if type(self.max_tokens) is not int or self.max_tokens < 1:
            raise ValueError("max_tokens must be an integer >= 1")
        if type(self.num_beams) is not int or self.num_beams < 1:
            raise ValueError("num_beams must be an integer >= 1")
        if self.no_repeat_ngram_size < 0 or self.min_length < 0:
            raise ValueError("no_repeat_ngram_size and min_length must be >= 0")
        if not self.repetition_penalty > 0:
            raise ValueError("repetition_penalty must be positive")

    @classmethod
    def from_dict(cls, d: dict) -> "SamplingParams":
        known = {f for f in cls.__dataclass_fields__ if f != "extra"}
        return cls(**{k: v for k, v in d.items() if k in known and v is not None})

    def eos_ids(self) -> list[int]:
        e = self.eos_token_id
        if e is None:
            return []
        return [e] if isinstance(e, int) else sorted(set(e))

    def beams_to_keep(self) -> int:
        return max(2, 1 + len(self.eos_ids())) * self.num_beams


def _as_list(x):
    if x is None:
        return []
    return [x] if isinstance(x, int) else list(x)


class LogitsRules:
    """Applies the enabled rules to a [rows, vocab] float tensor in place."""

    def __init__(self, params: SamplingParams, vocab_size: int, device):
        self.p = params
        self.vocab = vocab_size
        self.max_length = 1 + params.max_tokens      # decoder start token + generated tokens
        self.begin_index = 1 + int(params.forced_bos_token_id is not None)
        keep = lambda ids: [i for i in ids if 0 <= i < vocab_size]  # noqa: E731
        self.eos = torch.tensor(keep(params.eos_ids()), dtype=torch.long, device=device)
        self.suppress = torch.tensor(keep(_as_list(params.suppress_tokens)), dtype=torch.long, device=device)
        self.begin_suppress = torch.tensor(keep(_as_list(params.begin_suppress_tokens)), dtype=torch.long,
                                           device=device)
        self.forced_bos = keep(_as_list(params.forced_bos_token_id))
        self.forced_eos = keep(_as_list(params.forced_eos_token_id))
        self.needs_history = params.repetition_penalty != 1.0 or params.no_repeat_ngram_size > 0
        # whether any rule can change a score (else the selection reads the raw logits)
        self.active = bool(self.needs_history or (params.min_length > 0 and self.eos.numel()) or self.forced_bos
                           or self.forced_eos or self.suppress.numel() or self.begin_suppress.numel())

    def __call__(self, scores: torch.Tensor, hist: torch.Tensor | None, lengths: torch.Tensor) -> torch.Tensor:
        """``scores`` [rows, vocab] float (modified in place). ``hist`` [rows, W] int32: row i's
        decoder tokens (start token first) in columns [0, lengths[i]), anything after; only read
        when a rule needs the history. ``lengths`` int64 [rows] on the same device."""
        p = self.p
        dev = scores.device
        if p.repetition_penalty != 1.0:  # every token already in the row's history, once
            cols = torch.arange(hist.shape[1], device=dev)
            real = cols.unsqueeze(0) < lengths.unsqueeze(1)          # [rows, W]
            # columns past a row's length repeat its first token, so they rewrite that token's
            # (identical) penalised score and nothing else; no host synchronisation
            tokens = torch.where(real, hist, hist[:, :1]).long()
            seen = scores.gather(1, tokens)
            scores.scatter_(1, tokens, torch.where(seen < 0, seen * p.repetition_penalty, seen / p.repetition_penalty))
        if p.no_repeat_ngram_size > 0:
            self._ban_repeated_ngrams(scores, hist, lengths)
        if p.min_length > 0 and self.eos.numel():
            short = (lengths < p.min_length).unsqueeze(1)
            scores[:, self.eos] = scores[:, self.eos].masked_fill(short, NEG_INF)
        if self.forced_bos:
            self._force(scores, lengths == 1, self.forced_bos)
        if self.forced_eos:
            self._force(scores, lengths == self.max_length - 1, self.forced_eos)
        if self.suppress.numel():
            scores[:, self.suppress] = NEG_INF
        if self.begin_suppress.numel():
            first = (lengths == self.begin_index).unsqueeze(1)
            scores[:, self.begin_suppress] = scores[:, self.begin_suppress].masked_fill(first, NEG_INF)
        return scores

    @staticmethod
    def _force(scores, rows_mask, ids):
        """Make ``ids`` the only choice of each masked row: score 0 for them, -inf else."""
        ids_t = torch.tensor(ids, device=scores.device)
        keep = rows_mask.unsqueeze(1)
        forced = torch.full_like(scores, NEG_INF)
        forced[:, ids_t] = 0.0
        scores.copy_(torch.where(keep, forced, scores))

    def _ban_repeated_ngrams(self, scores, hist, lengths):
        """Ban every token that would complete an n-gram already in the row's history (rows
        shorter than n - 1 tokens ban nothing)."""
        n = self.p.no_repeat_ngram_size
        W = hist.shape[1]
        if W < n:
            return
        dev = scores.device
        windows = hist.unfold(1, n, 1)                                   # [rows, W - n + 1, n]
        starts = torch.arange(W - n + 1, device=dev)
        inside = starts.unsqueeze(0) + n <= lengths.unsqueeze(1)         # window within the row
        tail_pos = (lengths.unsqueeze(1) - (n - 1) + torch.arange(n - 1, device=dev)).clamp(min=0)
        tail = hist.gather(1, tail_pos)                                  # last n - 1 tokens
        match = (windows[:, :, : n - 1] == tail.unsqueeze(1)).all(-1) & inside
        match &= (lengths + 1 >= n).unsqueeze(1)
        # -inf where a window matches, +inf (no change under min) elsewhere: no host sync
        ban = torch.full(match.shape, float("inf"), device=dev).masked_fill_(match, NEG_INF)
        scores.scatter_reduce_(1, windows[:, :, n - 1].long(), ban, reduce="amin")
