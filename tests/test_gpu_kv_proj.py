"""Fused encoder K/V projection + paged write (vfl_kv_proj_paged, tensor cores) against a plain
PyTorch fp32 reference of the same op: kv = hidden @ w_kv.T + bias, rounded to bf16, scattered
by slot into [num_blocks, H, block_size, D] pools (vflorence/engine/model_runner.py:248-259).

Token counts from 6144 up, with 256-multiple feature counts, run the 2-SM (cta_group::2)
kernel; smaller ones the one-CTA kernel. Tolerance: bf16, 2e-2 absolute plus one bf16 step
(2^-7 relative) - both sides round the same fp32 value after sums in different orders, so an
entry at a rounding boundary may differ by one step; at least 99 % of entries must be bit-equal."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _case(tokens, hidden_dim, heads, head_dim, block_size, seed, with_bias=True, skip_every=7):
    g = torch.Generator(device=DEV).manual_seed(seed)
    gc = torch.Generator().manual_seed(seed)
    hidden = torch.randn(tokens, hidden_dim, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(2 * heads * head_dim, hidden_dim, generator=g, device=DEV) / hidden_dim ** 0.5).to(torch.bfloat16)
    bias = torch.randn(2 * heads * head_dim, generator=g, device=DEV).to(torch.bfloat16) if with_bias else None
    num_blocks = -(-tokens // block_size) + 5
    slots = torch.randperm(num_blocks * block_size, generator=gc)[:tokens].to(torch.int64)
    if skip_every:
        slots[::skip_every] = -1  # padded positions
    kc = torch.randn(num_blocks, heads, block_size, head_dim, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    return hidden, w, bias, kc, vc, slots.to(DEV)


def _reference(hidden, w, bias, kc, vc, slots):
    kv = hidden.float() @ w.float().T
    if bias is not None:
        kv = kv + bias.float()
    kv = kv.to(torch.bfloat16)
    n, h, bs, d = kc.shape
    k, v = kv[:, : h * d].view(-1, h, d), kv[:, h * d:].view(-1, h, d)
    ek, ev = kc.clone(), vc.clone()
    keep = slots >= 0
    s = slots[keep]
    ek[s // bs, :, s % bs] = k[keep]
    ev[s // bs, :, s % bs] = v[keep]
    return ek, ev


@pytest.mark.parametrize("tokens,hidden_dim,heads,head_dim,block_size,with_bias", [
    (300, 1024, 16, 64, 16, True),     # Florence-2-large / BART-large text shape, ragged token count
    (1000, 768, 12, 64, 16, True),     # Florence-2-base
    (128, 1024, 16, 64, 32, False),    # one full tile, block 32, no bias
    (77, 64, 2, 32, 16, True),         # one K step, head_dim 32
    (5000, 1024, 16, 64, 16, True),    # one-CTA kernel, 256-feature tiles, several tiles per CTA
    (4500, 768, 12, 64, 16, False),    # one-CTA kernel over 1536 features
    (6322, 768, 12, 64, 16, False),    # 2-SM pair tiles (256 tokens x 256 features); the last
                                       # tile's second CTA has 50 tokens
    (6200, 1024, 16, 64, 16, True),    # pair tiles; the last tile's second CTA has no tokens
    (20000, 1024, 16, 64, 32, True),   # many tiles per pair: both accumulators reused
])
def test_kv_proj_paged_matches_fp32_reference(tokens, hidden_dim, heads, head_dim, block_size, with_bias):
    from vflorence_b200 import paged_ops as ops

    hidden, w, bias, kc, vc, slots = _case(tokens, hidden_dim, heads, head_dim, block_size, seed=tokens,
                                           with_bias=with_bias)
    ek, ev = _reference(hidden, w, bias, kc, vc, slots)
    ops.kv_proj_paged(hidden, w, bias, kc, vc, slots)
    torch.cuda.synchronize()
    assert ops.read_device_errors(DEV) == 0
    for got, want, name in ((kc, ek, "k"), (vc, ev, "v")):
        diff = (got.float() - want.float()).abs()
        bound = 2e-2 + want.float().abs() * 2.0 ** -7
        assert bool((diff <= bound).all()), f"{name}: max |diff| {float(diff.max())}"
        assert float((diff == 0).float().mean()) >= 0.99, f"{name}: too few bit-equal entries"


def test_kv_proj_paged_equals_gemm_then_append():
    """The fused launch and the two-step path (cuBLAS GEMM, then the append kernel) agree."""
    from vflorence_b200 import paged_ops as ops

    hidden, w, bias, kc, vc, slots = _case(513, 1024, 16, 64, 16, seed=3)
    kc2, vc2 = kc.clone(), vc.clone()
    ops.kv_proj_paged(hidden, w, bias, kc, vc, slots)
    kv = torch.nn.functional.linear(hidden, w, bias)
    k, v = kv.chunk(2, dim=-1)
    ops.reshape_and_cache(k.reshape(-1, 16, 64), v.reshape(-1, 16, 64), kc2, vc2, slots)
    torch.cuda.synchronize()
    for got, want in ((kc, kc2), (vc, vc2)):
        assert bool(((got.float() - want.float()).abs() <= 2e-2 + want.float().abs() * 2.0 ** -7).all())


@pytest.mark.parametrize("tokens", [40, 7000], ids=["one_cta", "pair"])
def test_kv_proj_paged_flags_slots_past_the_pool(tokens):
    from vflorence_b200 import _native
    from vflorence_b200 import paged_ops as ops

    hidden, w, bias, kc, vc, slots = _case(tokens, 128, 2, 64, 16, seed=9, skip_every=0)
    before_k, before_v = kc.clone(), vc.clone()
    slots[5] = kc.shape[0] * kc.shape[2]  # one past the last slot: flagged, not written
    ek, ev = _reference(hidden, w, bias, before_k, before_v, torch.where(slots == slots[5], -1, slots))
    ops.kv_proj_paged(hidden, w, bias, kc, vc, slots)
    assert ops.read_device_errors(DEV) & _native.DEVERR_SLOT
    for got, want in ((kc, ek), (vc, ev)):
        assert bool(((got.float() - want.float()).abs() <= 2e-2 + want.float().abs() * 2.0 ** -7).all())


def test_kv_proj_paged_rejects_unbuilt_shapes():
    from vflorence_b200._native import VflError
    from vflorence_b200 import paged_ops as ops

    hidden, w, bias, kc, vc, slots = _case(16, 96, 2, 64, 16, seed=1)  # hidden_dim not a multiple of 64
    with pytest.raises(VflError):
        ops.kv_proj_paged(hidden, w, bias, kc, vc, slots)
