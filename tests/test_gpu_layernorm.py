"""Fused residual add + LayerNorm (vfl_add_layernorm) against a plain PyTorch fp32 reference of
the same op: out = LayerNorm(round(h + x)) * weight + bias, the decoder's post-norm residual
(vflorence/models/bart.py:192-201). Tolerances: fp32 1e-5 relative (plus 1e-5 absolute near
zero); bf16 2e-2 absolute. In bf16 the result must also equal torch's own add + LayerNorm
modules on at least 99 % of entries (both round the same fp32 value; the statistics are summed
in different orders)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _inputs(rows, d, dtype, seed, with_bias=True, strided=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    wide = 2 * d if strided else d
    h = (torch.randn(rows, wide, generator=g, device=DEV) * 3 + 0.5).to(dtype)[:, :d]
    x = torch.randn(rows, wide, generator=g, device=DEV).to(dtype)[:, wide - d:]
    w = (1 + 0.1 * torch.randn(d, generator=g, device=DEV)).to(dtype)
    b = (0.1 * torch.randn(d, generator=g, device=DEV)).to(dtype) if with_bias else None
    return h, x, w, b


def _reference(h, x, w, b, eps):
    s = (h + x).float()  # rounded to the dtype by the add, as the modules do
    return F.layer_norm(s, (s.shape[1],), w.float(), None if b is None else b.float(), eps)


@pytest.mark.parametrize("dtype,d", [(torch.bfloat16, 256), (torch.bfloat16, 768), (torch.bfloat16, 1024),
                                     (torch.bfloat16, 2048), (torch.float32, 128), (torch.float32, 768),
                                     (torch.float32, 1024)])
@pytest.mark.parametrize("rows", [1, 3, 255, 1000])
def test_add_layernorm_matches_fp32_reference(dtype, d, rows):
    from vflorence_b200 import paged_ops as ops

    h, x, w, b = _inputs(rows, d, dtype, seed=rows * 7 + d)
    out = ops.add_layernorm(h, x, w, b, 1e-5)
    ref = _reference(h, x, w, b, 1e-5)
    if dtype == torch.float32:
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
    else:
        assert float((out.float() - ref).abs().max()) <= 2e-2
        mods = F.layer_norm(h + x, (d,), w, b, 1e-5)
        assert float((out == mods).float().mean()) >= 0.99


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_add_layernorm_strided_rows_no_bias_and_in_place(dtype):
    from vflorence_b200 import paged_ops as ops

    d = 1024
    h, x, w, _ = _inputs(37, d, dtype, seed=3, with_bias=False, strided=True)
    assert h.stride(0) == 2 * d and x.stride(0) == 2 * d
    ref = _reference(h, x, w, None, 1e-6)
    out = ops.add_layernorm(h, x, w, None, 1e-6)
    tol = dict(rtol=1e-5, atol=1e-5) if dtype == torch.float32 else dict(rtol=0, atol=2e-2)
    torch.testing.assert_close(out.float(), ref, **tol)
    h2 = h.contiguous()
    same = ops.add_layernorm(h2, x, w, None, 1e-6, out=h2)  # the result replaces h
    assert same.data_ptr() == h2.data_ptr()
    torch.testing.assert_close(h2, out, rtol=0, atol=0)


def test_add_layernorm_rejects_unbuilt_widths():
    from vflorence_b200 import paged_ops as ops
    from vflorence_b200._native import VflError

    assert not ops.add_layernorm_supported(torch.bfloat16, 640)
    h, x, w, b = _inputs(4, 640, torch.bfloat16, seed=1)
    with pytest.raises(VflError):
        ops.add_layernorm(h, x, w, b, 1e-5)
