"""vfl_attention_with_kv_cache_no_alloc: the attention entry point for callers that cannot
allocate device memory (a C/C++ or FFI host without a device allocator, or a process whose
device memory a framework's pool already holds). Its split-K scratch is a fixed array inside
the library. Checked through the C ABI against vfl_attention_with_kv_cache with a caller-
provided workspace, on two calls in a row (the second call finds the first call's leftovers in
the shared scratch), and for the up-front rejection of plans that need more scratch than the
array holds. This file is collected last so that a failure here comes after every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import assert_attention_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
H, D, BS = 16, 64, 16


def _case(seed, num_reqs, min_len, max_len):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(min_len, max_len + 1, (num_reqs,), generator=g, dtype=torch.int32)
    need = [-(-int(n) // BS) for n in lens]
    nb = sum(need) + 2
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    table = torch.zeros(num_reqs, max(need), dtype=torch.int32)
    pos = 0
    for r, k in enumerate(need):
        table[r, :k] = perm[pos:pos + k]
        pos += k
    gd = torch.Generator(device=DEV).manual_seed(seed)
    kc = torch.randn(nb, H, BS, D, generator=gd, device=DEV, dtype=torch.bfloat16)
    vc = torch.randn(nb, H, BS, D, generator=gd, device=DEV, dtype=torch.bfloat16)
    q = torch.randn(num_reqs, H, D, generator=gd, device=DEV, dtype=torch.bfloat16)
    qsl = torch.arange(num_reqs + 1, dtype=torch.int32)
    return q, kc, vc, qsl, lens, table


def _run(lib, entry, plan, q, kc, vc, qsl, lens, table, ws=None):
    from vflorence_b200 import _native

    out = torch.full_like(q, float("nan"))
    args = [ctypes.byref(plan), q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), kc.shape[0],
            out.data_ptr(), out.stride(0), qsl.data_ptr(), lens.data_ptr(), table.data_ptr(),
            table.stride(0), table.shape[1], D ** -0.5]
    if entry == "vfl_attention_with_kv_cache":
        args += [ws.data_ptr(), ws.numel()]
    args.append(torch.cuda.current_stream(DEV).cuda_stream)
    _native.check(getattr(lib, entry)(*args), entry)
    return out


def test_no_alloc_matches_workspace_entry_point_twice(native):
    from vflorence_b200 import paged_ops as ops

    for call, (seed, n, lo, hi) in enumerate([(21, 3, 2000, 4096), (22, 5, 600, 3000)]):
        q, kc, vc, qsl, lens, table = _case(seed, n, lo, hi)
        meta = ops.get_scheduler_metadata(n, H, H, D, lens, torch.bfloat16, qsl, False, "sm100", BS)
        plan = ops.plan_of(meta)
        assert plan.num_splits > 1 and 0 < plan.workspace_bytes <= 64 * 1024 * 1024  # uses the scratch
        d = dict(qsl=qsl.to(DEV), lens=lens.to(DEV), table=table.to(DEV))
        ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=DEV)
        want = _run(native, "vfl_attention_with_kv_cache", plan, q, kc, vc, d["qsl"], d["lens"], d["table"], ws)
        got = _run(native, "vfl_attention_with_kv_cache_no_alloc", plan, q, kc, vc, d["qsl"], d["lens"],
                   d["table"])
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert_attention_close(got, want, torch.bfloat16, f"no-alloc call {call + 1}")
    assert ops.read_device_errors(DEV) == 0


def test_no_alloc_in_kernel_merge_counters_start_clean(native):
    """A caller-built plan that merges split partials inside the launch keeps arrival counters in
    the shared scratch; each call clears them first, so two calls in a row (the second finding
    the first's counters) both equal the workspace entry point."""
    from vflorence_b200 import _native
    from vflorence_b200 import paged_ops as ops

    for call, seed in enumerate((31, 32)):
        q, kc, vc, qsl, lens, table = _case(seed, 4, 1500, 4096)
        meta = ops.get_scheduler_metadata(4, H, H, D, lens, torch.bfloat16, qsl, False, "sm100", BS)
        planned = ops.plan_of(meta)
        plan = _native.AttentionPlan()
        ctypes.memmove(ctypes.byref(plan), ctypes.byref(planned), ctypes.sizeof(plan))
        assert plan.num_splits > 1 and plan.merge_in_kernel == 0
        groups = H // plan.heads_per_cta
        q_chunks = -(-plan.max_q_len // plan.queries_per_cta)
        plan.merge_in_kernel = 1
        plan.workspace_bytes += plan.num_reqs * groups * q_chunks * 4  # the arrival counters
        d = dict(qsl=qsl.to(DEV), lens=lens.to(DEV), table=table.to(DEV))
        ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=DEV)
        want = _run(native, "vfl_attention_with_kv_cache", plan, q, kc, vc, d["qsl"], d["lens"], d["table"], ws)
        got = _run(native, "vfl_attention_with_kv_cache_no_alloc", plan, q, kc, vc, d["qsl"], d["lens"],
                   d["table"])
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert_attention_close(got, want, torch.bfloat16, f"in-kernel merge, no-alloc call {call + 1}")
    assert ops.read_device_errors(DEV) == 0


def test_no_alloc_balanced_plans_twice(native):
    """Balanced plans keep their partial records and item directory in the shared scratch; two
    calls in a row with other lengths (the second finding the first's directory there) both
    equal the workspace entry point."""
    from vflorence_b200 import paged_ops as ops

    for call, (seed, n, lo, hi) in enumerate([(41, 40, 1, 4096), (42, 24, 1500, 2000)]):
        q, kc, vc, qsl, lens, table = _case(seed, n, lo, hi)
        meta = ops.get_scheduler_metadata(n, H, H, D, lens, torch.bfloat16, qsl, False, "sm100", BS)
        plan = ops.plan_of(ops.set_schedule(meta, ops.SCHEDULE_BALANCED))
        assert 0 < plan.workspace_bytes <= 64 * 1024 * 1024
        d = dict(qsl=qsl.to(DEV), lens=lens.to(DEV), table=table.to(DEV))
        ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=DEV)
        want = _run(native, "vfl_attention_with_kv_cache", plan, q, kc, vc, d["qsl"], d["lens"], d["table"], ws)
        got = _run(native, "vfl_attention_with_kv_cache_no_alloc", plan, q, kc, vc, d["qsl"], d["lens"],
                   d["table"])
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert torch.equal(got, want), f"balanced, no-alloc call {call + 1}"  # same plan, same sums
    assert ops.read_device_errors(DEV) == 0


def test_no_alloc_rejects_plans_beyond_its_scratch(native):
    from vflorence_b200 import _native
    from vflorence_b200 import paged_ops as ops

    lens = torch.full((4096,), 4096, dtype=torch.int32)
    meta = ops.get_scheduler_metadata(4096, H, H, D, lens, torch.bfloat16, None, False, "sm100", BS)
    plan = ops.plan_of(meta)
    assert plan.workspace_bytes > _native.STATIC_WORKSPACE_BYTES
    st = native.vfl_attention_with_kv_cache_no_alloc(ctypes.byref(plan), None, 0, None, None, 0, None, 0,
                                                      None, None, None, 0, 0, 1.0, None)
    assert st == _native.VFL_ERR_WORKSPACE
    assert b"built-in scratch" in native.vfl_last_error_message()
