"""The host decode runtime (``include/vflorence_b200_runtime.h``) bound over ctypes.

One ``DecodeRuntime`` owns a self-attention block pool's bookkeeping and the decode
hypotheses of an engine: block tables, reference counts, the free list, the running list and
every request's finished hypotheses. Each step the engine makes a handful of calls:

    admit          new requests enter the running list
    prepare_step   room for every row's next token; copy-on-write pairs
    pack_step      the rows' step inputs written straight into (pinned) numpy buffers
    advance_*      the step's decisions from the device's picks or beam candidates

All arrays cross as plain pointers into numpy buffers; nothing here touches the GPU.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _native as N


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


@dataclass
class StepRows:
    """The running rows of a step (numpy views, valid until the next pack)."""

    n: int
    table_lens: np.ndarray    # int32 [n]
    positions: np.ndarray     # int32 [n]
    tokens: np.ndarray        # int32 [n]
    slots: np.ndarray         # int32 [n]
    lengths: np.ndarray       # int32 [n]
    request_ids: np.ndarray   # int64 [n]
    groups: np.ndarray        # int32 [n]
    ranks: np.ndarray         # int32 [n]
    cum_logprobs: np.ndarray  # float32 [n]
    num_groups: int
    max_rank: int


@dataclass
class StepResult:
    """A step's decisions (numpy copies)."""

    born_parent: np.ndarray
    born_child: np.ndarray
    born_pos: np.ndarray
    born_token: np.ndarray
    done_request: np.ndarray
    done_slot: np.ndarray
    done_length: np.ndarray


class DecodeRules:
    """The decoding parameters the host bookkeeping needs, as a ``vfl_decode_rules``."""

    def __init__(self, num_beams: int, max_tokens: int, length_penalty: float, early_stopping: bool,
                 eos_ids):
        self._eos = np.ascontiguousarray(np.asarray(list(eos_ids), dtype=np.int32))
        self.c = N.DecodeRules(int(num_beams), int(max_tokens), float(length_penalty), int(bool(early_stopping)),
                               len(self._eos), self._eos.ctypes.data if len(self._eos) else None)

    @classmethod
    def from_params(cls, params) -> "DecodeRules":
        return cls(params.num_beams, params.max_tokens, params.length_penalty, params.early_stopping,
                   params.eos_ids())


class DecodeRuntime:
    def __init__(self, num_blocks: int, block_size: int, num_slots: int, max_blocks_per_seq: int):
        self._lib = N.lib()
        h = ctypes.c_void_p()
        N.check(self._lib.vfl_rt_create(num_blocks, block_size, num_slots, max_blocks_per_seq, ctypes.byref(h)),
                "runtime create")
        self._h = h
        self.num_blocks, self.block_size = num_blocks, block_size
        self.num_slots, self.max_blocks_per_seq = num_slots, max_blocks_per_seq
        i32 = lambda k: np.zeros(k, dtype=np.int32)  # noqa: E731
        S = num_slots
        self._pairs = i32(2 * S)
        self._i32 = {name: i32(S) for name in ("table_lens", "positions", "tokens", "slots", "lengths", "groups",
                                                "ranks")}
        self._rids = np.zeros(S, dtype=np.int64)
        self._cum = np.zeros(S, dtype=np.float32)
        self._born = [i32(S) for _ in range(4)]
        self._done_rid = np.zeros(S, dtype=np.int64)
        self._done = [i32(S) for _ in range(2)]
        self._out = ctypes.c_int32()
        self._out2 = ctypes.c_int32()
        self._res = N.StepResult(*(b.ctypes.data for b in self._born), S, 0, self._done_rid.ctypes.data,
                                 self._done[0].ctypes.data, self._done[1].ctypes.data, S, 0)
        # the per-step output buffers live as long as the runtime: their addresses are taken once
        # (numpy's .ctypes.data costs about 2 us a call, and a step passes a dozen of them)
        self._addr = {name: a.ctypes.data for name, a in self._i32.items()}
        self._addr_rids, self._addr_cum = self._rids.ctypes.data, self._cum.ctypes.data
        self._ng, self._mr = ctypes.c_int32(), ctypes.c_int32()

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self._lib.vfl_rt_destroy(h)
            self._h = None

    def _check(self, status: int, what: str) -> None:
        if status != N.VFL_OK:
            N.check(status, what)

    # ------------------------------------------------------------------------ block manager
    def reset(self) -> None:
        self._check(self._lib.vfl_rt_reset(self._h), "runtime reset")

    def slot_acquire(self) -> int:
        self._check(self._lib.vfl_rt_slot_acquire(self._h, ctypes.byref(self._out)), "slot_acquire")
        return self._out.value

    def slot_release(self, slot: int) -> None:
        self._check(self._lib.vfl_rt_slot_release(self._h, slot), "slot_release")

    @property
    def num_free_blocks(self) -> int:
        self._check(self._lib.vfl_rt_num_free_blocks(self._h, ctypes.byref(self._out)), "num_free_blocks")
        return self._out.value

    def free_block_ids(self) -> list[int]:
        buf = np.zeros(self.num_blocks, dtype=np.int32)
        self._check(self._lib.vfl_rt_free_block_ids(self._h, buf.ctypes.data, self.num_blocks,
                                                     ctypes.byref(self._out)), "free_block_ids")
        return buf[: self._out.value].tolist()

    def ref_count(self, block: int) -> int:
        self._check(self._lib.vfl_rt_ref_count(self._h, block, ctypes.byref(self._out)), "ref_count")
        return self._out.value

    def ref_counts(self) -> list[int]:
        return [self.ref_count(b) for b in range(self.num_blocks)]

    def block_table(self, slot: int) -> list[int]:
        buf = np.zeros(self.max_blocks_per_seq, dtype=np.int32)
        self._check(self._lib.vfl_rt_block_table(self._h, slot, buf.ctypes.data, self.max_blocks_per_seq,
                                                  ctypes.byref(self._out)), "block_table")
        return buf[: self._out.value].tolist()

    def required_new_blocks(self, slots, num_cached) -> int:
        s = np.ascontiguousarray(slots, dtype=np.int32)
        c = np.ascontiguousarray(num_cached, dtype=np.int32)
        out = ctypes.c_int64()
        self._check(self._lib.vfl_rt_required_new_blocks(self._h, _ptr(s), _ptr(c), len(s), ctypes.byref(out)),
                    "required_new_blocks")
        return out.value

    def ensure_capacity(self, slot: int, num_cached: int) -> tuple[int, int] | None:
        self._check(self._lib.vfl_rt_ensure_capacity(self._h, slot, num_cached, ctypes.byref(self._out),
                                                      ctypes.byref(self._out2)), "ensure_capacity")
        return None if self._out.value < 0 else (self._out.value, self._out2.value)

    def fork(self, parent: int, child: int) -> None:
        self._check(self._lib.vfl_rt_fork(self._h, parent, child), "fork")

    def deallocate(self, slot: int) -> None:
        self._check(self._lib.vfl_rt_deallocate(self._h, slot), "deallocate")

    # ---------------------------------------------------------------------- decode rows
    def admit(self, request_id: int, start_token: int) -> int:
        self._check(self._lib.vfl_rt_admit(self._h, request_id, start_token, ctypes.byref(self._out)), "admit")
        return self._out.value

    @property
    def num_running(self) -> int:
        self._check(self._lib.vfl_rt_num_running(self._h, ctypes.byref(self._out)), "num_running")
        return self._out.value

    def prepare_step(self) -> np.ndarray:
        """Copy-on-write pairs of the step, int32 [P, 2] (a view, valid until the next call)."""
        self._check(self._lib.vfl_rt_prepare_step(self._h, self._pairs.ctypes.data, self.num_slots,
                                                   ctypes.byref(self._out)), "prepare_step")
        return self._pairs[: 2 * self._out.value].reshape(-1, 2)

    def pack_step(self, tables: np.ndarray | None = None, positions: np.ndarray | None = None,
                  tokens: np.ndarray | None = None) -> StepRows:
        """The running rows' inputs. ``tables`` ([>= n, width] int32, row-contiguous),
        ``positions`` and ``tokens`` may be caller buffers (e.g. a pinned upload buffer)."""
        a = self._i32
        pos = a["positions"] if positions is None else positions
        tok = a["tokens"] if tokens is None else tokens
        if tables is not None:
            if tables.dtype != np.int32 or tables.ndim != 2 or tables.strides[1] != 4:
                raise ValueError("pack_step: tables must be a row-contiguous int32 [rows, width] array")
            stride, width = tables.strides[0] // 4, tables.shape[1]
            cap = tables.shape[0]
        else:
            stride, width, cap = 0, 0, self.num_slots
        cap = min(cap, len(pos), len(tok))
        ad, ng, mr = self._addr, self._ng, self._mr
        self._check(self._lib.vfl_rt_pack_step(
            self._h, cap, _ptr(tables), stride, width, ad["table_lens"],
            ad["positions"] if positions is None else _ptr(pos), ad["tokens"] if tokens is None else _ptr(tok),
            ad["slots"], ad["lengths"], self._addr_rids, ad["groups"], ad["ranks"], self._addr_cum,
            ctypes.byref(ng), ctypes.byref(mr)), "pack_step")
        n = self.num_running
        return StepRows(n, a["table_lens"][:n], pos[:n], tok[:n], a["slots"][:n], a["lengths"][:n], self._rids[:n],
                        a["groups"][:n], a["ranks"][:n], self._cum[:n], ng.value, mr.value)

    def _result(self) -> StepResult:
        nb, nd = self._res.num_born, self._res.num_done
        b = [x[:nb].copy() for x in self._born]
        return StepResult(*b, self._done_rid[:nd].copy(), self._done[0][:nd].copy(), self._done[1][:nd].copy())

    def advance_greedy(self, rules: DecodeRules, picks: np.ndarray) -> StepResult:
        p = np.ascontiguousarray(picks, dtype=np.int64)
        self._check(self._lib.vfl_rt_advance_greedy(self._h, ctypes.byref(rules.c), p.ctypes.data, len(p),
                                                     ctypes.byref(self._res)), "advance_greedy")
        return self._result()

    def advance_beam(self, rules: DecodeRules, rows: np.ndarray, tokens: np.ndarray, scores: np.ndarray) -> StepResult:
        """``rows``/``tokens`` int32 and ``scores`` float32, each [num_groups, per_group]."""
        r = np.ascontiguousarray(rows, dtype=np.int32)
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        s = np.ascontiguousarray(scores, dtype=np.float32)
        if r.ndim != 2 or r.shape != t.shape or r.shape != s.shape:
            raise ValueError("advance_beam: candidates must be three [num_groups, per_group] arrays")
        cap = max(self.num_slots, r.size)
        if cap > len(self._born[0]):
            self._grow_results(cap)
        self._check(self._lib.vfl_rt_advance_beam(self._h, ctypes.byref(rules.c), r.ctypes.data, t.ctypes.data,
                                                   s.ctypes.data, r.shape[0], r.shape[1], ctypes.byref(self._res)),
                    "advance_beam")
        return self._result()

    def _grow_results(self, cap: int) -> None:
        self._born = [np.zeros(cap, dtype=np.int32) for _ in range(4)]
        self._res.born_parent, self._res.born_child, self._res.born_pos, self._res.born_token = (
            b.ctypes.data for b in self._born)
        self._res.born_cap = cap
