"""decode_linear (the float32 linear layer of a decode step of <= 16 rows) against a float64
reference of the same op, at the fp32 parity bar; exact GELU; fixed reduction order (bitwise
repeatable); strided rows."""

from __future__ import annotations

import math

import pytest
import torch

from conftest import assert_attention_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

# (n, k): BART-large decoder layers (q/k/v, out, fc1, fc2), the padded vocabulary projection,
# and the golden-trace / tiny Florence-2 widths
SHAPES = [(3072, 1024), (1024, 1024), (4096, 1024), (1024, 4096), (50304, 1024), (384, 128), (96, 256)]


def _reference(x, w, b, gelu):
    y = x.double() @ w.double().T
    if b is not None:
        y = y + b.double()
    if gelu:
        y = 0.5 * y * (1.0 + torch.erf(y / math.sqrt(2.0)))
    return y


@pytest.mark.parametrize("rows", [1, 3, 8, 16])
@pytest.mark.parametrize("n,k", SHAPES)
def test_decode_linear_matches_float64(rows, n, k):
    from vflorence_b200 import paged_ops as ops

    assert ops.decode_linear_supported(torch.float32, rows, n, k)
    g = torch.Generator(device=DEV).manual_seed(n * 7 + k + rows)
    x = torch.randn(rows, k, device=DEV, generator=g)
    w = torch.randn(n, k, device=DEV, generator=g) * 0.02
    b = torch.randn(n, device=DEV, generator=g)
    for bias, gelu in ((b, False), (None, False), (b, True)):
        y = ops.decode_linear(x, w, bias, "gelu" if gelu else None)
        assert_attention_close(y, _reference(x, w, bias, gelu), torch.float32, f"rows {rows} n {n} k {k}")
    assert ops.read_device_errors(DEV) == 0


def test_decode_linear_is_repeatable_and_takes_strided_rows():
    from vflorence_b200 import paged_ops as ops

    g = torch.Generator(device=DEV).manual_seed(1)
    wide = torch.randn(8, 1024 + 64, device=DEV, generator=g)
    x = wide[:, 32:32 + 1024]  # row stride 1088, 16-byte aligned start
    w = torch.randn(1024, 1024, device=DEV, generator=g)
    b = torch.randn(1024, device=DEV, generator=g)
    out = torch.zeros(8, 1024 + 32, device=DEV)
    y1 = ops.decode_linear(x, w, b)
    y2 = ops.decode_linear(x, w, b, out=out[:, :1024])
    assert torch.equal(y1, y2) and torch.equal(y1, ops.decode_linear(x.contiguous(), w, b))
    assert bool((out[:, 1024:] == 0).all())
    assert_attention_close(y1, _reference(x, w, b, False), torch.float32, "strided")
