"""Failure detection on the GPU without a fault: a bounded wait made to run out.

``vfl_check_bounded_wait`` runs the shared-memory barrier wait of the pipelined kernels on its own:
the consumer warp waits for an arrival that the producer warp withholds (a flag nothing sets).
The wait must give up after its short limit, the kernel must exit, the device error word must
read VFL_DEVERR_TIMEOUT, and the GPU must keep answering: the next calls, attention included,
run normally. Nothing here faults, traps or hangs a GPU: the wait is bounded by a 1 ms limit.
"""

from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_withheld_arrival_times_out_and_reports(oracle_lib):
    from vflorence_b200 import _native as N
    from vflorence_b200 import paged_ops as ops

    assert ops.read_device_errors(DEV) == 0
    t0 = time.perf_counter()
    ops.check_bounded_wait(1_000_000, producer_arrives=False, device=DEV)  # 1 ms limit
    bits = ops.read_device_errors(DEV)  # synchronises: the kernel has exited
    elapsed = time.perf_counter() - t0
    assert bits == N.DEVERR_TIMEOUT
    assert elapsed < 1.0  # gave up after its limit, not the 2 s default
    assert ops.read_device_errors(DEV) == 0  # read cleared the word

    # the same wait with the arrival made: no error
    ops.check_bounded_wait(1_000_000, producer_arrives=True, device=DEV)
    assert ops.read_device_errors(DEV) == 0

    # the context is still usable: an attention call right after matches the oracle
    g = torch.Generator().manual_seed(4)
    H, D, bs, nb = 4, 64, 16, 24
    kc = torch.randn(nb, H, bs, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(nb, H, bs, D, generator=g).to(torch.bfloat16)
    q = torch.randn(2, H, D, generator=g).to(torch.bfloat16)
    lens = torch.tensor([100, 37], dtype=torch.int32)
    qsl = torch.arange(3, dtype=torch.int32)
    table = torch.randperm(nb, generator=g)[:14].to(torch.int32).view(2, 7)
    meta = ops.get_scheduler_metadata(2, H, H, D, lens, torch.bfloat16, qsl, False, "sm100", bs)
    out = torch.empty_like(q, device=DEV)
    ops.attention_with_kv_cache(q.to(DEV), kc.to(DEV), vc.to(DEV), out, qsl.to(DEV), lens.to(DEV), D ** -0.5,
                                False, table.to(DEV), meta)
    want = torch.empty_like(q)
    oracle_lib.attention(q, kc, vc, want, qsl, lens, D ** -0.5, False, table)
    assert ops.read_device_errors(DEV) == 0
    assert (out.float().cpu() - want.float()).abs().max().item() <= 2e-2


def test_timeout_bit_stops_later_attention_launches_until_cleared():
    """While VFL_DEVERR_TIMEOUT is set, attention CTAs exit at once (an earlier wait gave up, so
    later work is not trusted); after the read clears it, the same call computes again."""
    from vflorence_b200 import _native as N
    from vflorence_b200 import paged_ops as ops

    H, D, bs = 4, 64, 16
    kc = torch.randn(8, H, bs, D, device=DEV).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    q = torch.randn(1, H, D, device=DEV).to(torch.bfloat16)
    lens = torch.tensor([40], dtype=torch.int32)
    qsl = torch.arange(2, dtype=torch.int32)
    table = torch.tensor([[3, 1, 6]], dtype=torch.int32, device=DEV)
    meta = ops.get_scheduler_metadata(1, H, H, D, lens, torch.bfloat16, qsl, False, "sm100", bs)

    def attend():
        out = torch.full_like(q, 7.0)
        ops.attention_with_kv_cache(q, kc, vc, out, qsl.to(DEV), lens.to(DEV), D ** -0.5, False, table, meta)
        return out

    ops.check_bounded_wait(1_000_000, producer_arrives=False, device=DEV)
    skipped = attend()
    assert ops.read_device_errors(DEV) == N.DEVERR_TIMEOUT
    assert bool((skipped == 7.0).all())  # nothing written while the bit was set
    computed = attend()
    assert ops.read_device_errors(DEV) == 0
    assert not bool((computed == 7.0).any())
