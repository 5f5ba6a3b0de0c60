"""Shared fixtures. GPU tests carry @pytest.mark.gpu; the CPU suite runs with -m "not gpu"."""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (REPO, os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def native():
    from vflorence_b200 import build

    build.build()
    from vflorence_b200 import _native

    return _native.lib()


@pytest.fixture(scope="session")
def engine_trace():
    return torch.load(os.path.join(GOLDEN, "engine_trace.pt"), weights_only=True)


def load_attention_cases():
    z = np.load(os.path.join(GOLDEN, "attention_cases.npz"))
    cases = []
    for i in range(int(z["num_cases"])):
        c = {k.split(":", 1)[1]: z[k] for k in z.files if k.startswith(f"{i}:")}
        for k in ("name", "dtype"):
            c[k] = str(c[k])
        for k in ("causal", "block_size"):
            c[k] = int(c[k])
        c["scale"] = float(c["scale"])
        cases.append(c)
    return cases


def bf16_from_bits(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


def case_tensors(c, dtype=None):
    """Tensors of an attention case in its dtype (or ``dtype``)."""
    dt = dtype or (torch.float32 if c["dtype"] == "f32" else torch.bfloat16)
    t = {k: bf16_from_bits(c[k]).to(dt) for k in ("q", "k_cache", "v_cache")}
    for k in ("query_start_loc", "seq_lens", "block_table"):
        t[k] = torch.from_numpy(c[k].astype(np.int32))
    t["expected"] = torch.from_numpy(c["expected"])
    return t


def assert_attention_close(got: torch.Tensor, want: torch.Tensor, dtype: torch.dtype, what=""):
    """The parity bar for attention outputs.

    float32: |got - want| <= 1e-5 * |want| + 1e-5 * max|want|   (1e-5 relative, scaled to the
             output's magnitude so that entries near zero are not held to a relative bound)
    bfloat16: |got - want| <= 2e-2 absolute
    """
    got, want = got.double().cpu(), want.double().cpu()
    if dtype == torch.float32:
        scale = want.abs().max().item() if want.numel() else 0.0
        tol = 1e-5 * want.abs() + 1e-5 * scale
    else:
        tol = torch.full_like(want, 2e-2)
    diff = (got - want).abs()
    bad = diff > tol
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.numel()} entries outside tolerance; "
                           f"max|diff| {diff.max().item():.3e}")
