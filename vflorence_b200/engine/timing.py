"""Where a decode job's time goes: CUDA-event intervals per phase on the engine's stream.

A ``PhaseTimer`` given to the engine brackets the vision tower, the text encoder, the encoder
K/V paging and every whole step with event pairs; nothing synchronises during the job. After
the job (and a synchronize), ``summary()`` sums each phase in milliseconds of the stream's
timeline - kernels plus any idle gaps inside the bracket, so host-bound stretches count where
they happen. ``decode`` is the steps' time minus the encoder phases that ran inside them.
"""

from __future__ import annotations

from contextlib import contextmanager

import torch


class PhaseTimer:
    def __init__(self):
        self._events: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    @contextmanager
    def __call__(self, name: str):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        try:
            yield
        finally:
            end.record()
            self._events.append((name, start, end))

    def summary(self) -> dict[str, float]:
        """Milliseconds per phase (call after the stream has finished the job)."""
        out: dict[str, float] = {}
        counts: dict[str, int] = {}
        for name, start, end in self._events:
            out[name] = out.get(name, 0.0) + start.elapsed_time(end)
            counts[name] = counts.get(name, 0) + 1
        enc = sum(out.get(k, 0.0) for k in ("vision_tower", "text_encoder", "encoder_kv_pages"))
        if "step" in out:
            out["decode"] = out["step"] - enc
            out["steps"] = counts["step"]
        return out
