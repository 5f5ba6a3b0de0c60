"""Device candidate selection (vfl_row_topk, vfl_beam_merge) against plain PyTorch fp32: the
log_softmax / top-k / cumulative-log-prob add of the reference's _sample and _beam_search
(vflorence/engine/model_runner.py:370-410), with ties ordered by lower index (argmax's rule)
and the per-request merge ordered as a stable descending sort of the rows' lists."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _expected_topk(x: torch.Tensor, k: int, log_softmax: bool, offset):
    xf = x.float()
    order = torch.sort(xf, dim=1, descending=True, stable=True).indices[:, :k]   # ties: lower index first
    vals = torch.log_softmax(xf, dim=-1) if log_softmax else xf
    out = vals.gather(1, order)
    if offset is not None:
        out = out + offset.unsqueeze(1)
    return out, order


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("vocab,k", [(51289, 6), (50265, 8), (1000, 1), (777, 13), (4096, 32), (3000, 64), (5, 5)])
@pytest.mark.parametrize("log_softmax", [False, True])
def test_row_topk_matches_torch(dtype, vocab, k, log_softmax):
    from vflorence_b200 import paged_ops as ops

    g = torch.Generator(device=DEV).manual_seed(vocab + k)
    rows = 37
    x = (torch.randn(rows, vocab, generator=g, device=DEV) * 3).to(dtype)
    x[3, ::7] = float("-inf")
    offset = torch.randn(rows, generator=g, device=DEV) * 10
    vals, ids = ops.row_topk(x, k, log_softmax=log_softmax, row_offset=offset)
    want_v, want_i = _expected_topk(x, k, log_softmax, offset)
    assert torch.equal(ids.long(), want_i)
    torch.testing.assert_close(vals, want_v, rtol=0, atol=2e-5)


def test_row_topk_ties_and_strides():
    from vflorence_b200 import paged_ops as ops

    g = torch.Generator(device=DEV).manual_seed(5)
    # small integers: many equal values; rows of an odd length are not 16-byte aligned
    x = torch.randint(-4, 4, (64, 51289), generator=g, device=DEV).to(torch.bfloat16)
    for k in (1, 6, 16):
        _, ids = ops.row_topk(x, k)
        assert torch.equal(ids.long(), _expected_topk(x, k, False, None)[1])
    # a column slice of a wider matrix (row stride > vocab), as the padded vocabulary projection gives
    wide = torch.randn(16, 51328, generator=g, device=DEV).to(torch.bfloat16)
    view = wide[:, :51289]
    v, ids = ops.row_topk(view, 6, log_softmax=True)
    want_v, want_i = _expected_topk(view, 6, True, None)
    assert torch.equal(ids.long(), want_i)
    torch.testing.assert_close(v, want_v, rtol=0, atol=2e-5)
    # k = 1 is torch.argmax (first maximal index)
    _, ids = ops.row_topk(x, 1)
    assert torch.equal(ids.view(-1).long(), x.float().argmax(dim=-1))


def test_row_topk_rejects_bad_k():
    from vflorence_b200 import paged_ops as ops
    from vflorence_b200._native import VflError

    x = torch.zeros(2, 10, device=DEV)
    for k in (0, 11, 65):
        with pytest.raises(VflError):
            ops.row_topk(x, k)


def _torch_merge(values, ids, groups, ranks, R, keep):
    """The grid + stable sort formulation of the per-request merge."""
    n, k = values.shape
    width = int(ranks.max()) + 1
    grid_s = torch.full((R, width, k), float("-inf"), device=DEV)
    grid_t = torch.zeros((R, width, k), dtype=torch.int32, device=DEV)
    grid_r = torch.full((R, width, k), -1, dtype=torch.int32, device=DEV)
    gl, rl = groups.long(), ranks.long()
    grid_s[gl, rl] = values
    grid_t[gl, rl] = ids
    grid_r[gl, rl] = torch.arange(n, device=DEV, dtype=torch.int32).unsqueeze(-1).expand(n, k)
    srt, pos = torch.sort(grid_s.view(R, -1), dim=1, descending=True, stable=True)
    m = min(keep, width * k)
    rows = grid_r.view(R, -1).gather(1, pos[:, :m])
    toks = grid_t.view(R, -1).gather(1, pos[:, :m])
    return rows, toks, srt[:, :m]


@pytest.mark.parametrize("beams,k,keep", [(3, 6, 6), (4, 8, 8), (1, 2, 2), (8, 16, 16)])
@pytest.mark.parametrize("contiguous", [True, False])
def test_beam_merge_matches_stable_sort(beams, k, keep, contiguous):
    from vflorence_b200 import paged_ops as ops

    g = torch.Generator().manual_seed(beams * 31 + k)
    R = 23
    counts = torch.randint(1, beams + 1, (R,), generator=g).tolist()
    groups = torch.cat([torch.full((c,), r, dtype=torch.int32) for r, c in enumerate(counts)])
    ranks = torch.cat([torch.arange(c, dtype=torch.int32) for c in counts])
    if not contiguous:  # rows of a request need not be adjacent; ranks keep their order
        perm = torch.randperm(len(groups), generator=g)
        groups, ranks = groups[perm], ranks[perm]
        # re-rank by position so a group's ranks follow row order, as the runtime gives them
        for r in range(R):
            idx = (groups == r).nonzero().view(-1)
            ranks[idx] = torch.arange(len(idx), dtype=torch.int32)
    n = len(groups)
    # coarse values: many ties across rows and within lists
    values = (torch.randint(-6, 0, (n, k), generator=g).float() / 2).sort(dim=1, descending=True).values
    ids = torch.randint(0, 50000, (n, k), generator=g, dtype=torch.int32)
    values, ids, groups, ranks = (t.to(DEV) for t in (values, ids, groups, ranks))
    out = ops.beam_merge(values, ids, groups, ranks, R, keep).cpu()
    rows, toks, vals = (t.cpu() for t in _torch_merge(values, ids, groups, ranks, R, keep))
    m = rows.shape[1]
    for r in range(R):
        valid = rows[r] >= 0
        got = out[0, r][out[0, r] >= 0]
        assert torch.equal(got, rows[r][valid])
        assert torch.equal(out[1, r][: len(got)], toks[r][valid])
        assert torch.equal(out[2, r][: len(got)].view(torch.float32), vals[r][valid])
        assert (out[0, r][len(got):] == -1).all() and len(got) <= min(keep, m)


def test_fork_token_rows_matches_index_ops():
    """Children's token rows in one launch equal the two torch index ops they replace
    (Sequence.fork, vflorence/engine/sequence.py:53-55); bad rows are skipped and flagged."""
    from vflorence_b200 import _native
    from vflorence_b200 import paged_ops as ops

    g = torch.Generator().manual_seed(4)
    slots, width = 40, 1026
    tokens = torch.randint(0, 51289, (slots, width), generator=g, dtype=torch.int32).to(DEV)
    perm = torch.randperm(slots, generator=g)
    parents = perm[:10].repeat(2)[:17]                     # a parent may have several children
    children = perm[10:27]                                  # never a parent of the same step
    pos = torch.randint(0, width, (17,), generator=g)
    tok = torch.randint(0, 51289, (17,), generator=g)
    born = torch.stack([parents, children, pos, tok]).to(torch.int32).contiguous().to(DEV)
    want = tokens.clone()
    b = born.long()
    want[b[1]] = want[b[0]]
    want[b[1], b[2]] = b[3].to(torch.int32)
    ops.fork_token_rows(tokens, born)
    assert torch.equal(tokens, want)
    assert ops.read_device_errors(DEV) == 0
    bad = born[:, :2].clone()
    bad[1, 1] = slots  # a child row past the buffer: skipped, flagged
    before = tokens.clone()
    ops.fork_token_rows(tokens, bad)
    assert ops.read_device_errors(DEV) & _native.DEVERR_SLOT
    expect = before.clone()
    expect[bad[1, 0].long()] = before[bad[0, 0].long()]
    expect[bad[1, 0].long(), bad[2, 0].long()] = bad[3, 0]
    assert torch.equal(tokens, expect)
