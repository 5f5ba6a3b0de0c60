"""Decoder attention custom ops on B200 (mirror of vflorence/layers/attention.py:1-115).

The ops keep the reference's opaque ``torch.library.custom_op`` surface - same names
(``vflorence::self_attention``, ``vflorence::cross_attention``), same arguments, same fake
implementations - so a decoder compiled around them is unchanged. The work goes to the sm_100a
kernels through ``paged_ops`` instead of ``vllm_cpu_attn``.
"""

from __future__ import annotations

import torch

from . import paged_ops
from .context import get_context

HEAD_DIMS = paged_ops.HEAD_DIMS


def group_rows(pages, enc_lens):
    """Split running rows into runs that share one request's encoder pages.

    Beams of a request are consecutive rows with the same ``pages`` tensor (the runner keeps one
    tensor per request, vflorence/engine/model_runner.py:244-245). Returns
    (first row of each run, row offsets [runs + 1]).
    """
    firsts, offsets = [], []
    for i, (p, n) in enumerate(zip(pages, enc_lens)):
        if i == 0 or p is not pages[i - 1] or n != enc_lens[i - 1]:
            firsts.append(i)
            offsets.append(i)
    offsets.append(len(pages))
    return firsts, offsets


def stage_cross(layers, pages, enc_lens, block_size: int, isa: str):
    """Point this step's rows at their encoder K/V pages in each layer's pool; nothing is copied.

    ``pages[i]`` (int32 device tensor) and ``enc_lens[i]`` belong to running row i; beams of one
    request repeat its pages (vflorence/layers/attention.py:9-39). On B200 each run of rows that
    share pages becomes ONE request with several query rows, so the cross-attention kernel reads
    every encoder page once per request instead of once per beam. Each staged entry is
    ``(k_cache, v_cache, block_table, seq_lens, metadata, query_start_loc)``.
    """
    attn = layers[0].encoder_attn
    device = attn.k_cache.device
    firsts, offsets = group_rows(pages, enc_lens)
    group_pages = [pages[i] for i in firsts]
    width = max(1, max(int(p.numel()) for p in group_pages))
    on_host = all(p.device.type == "cpu" for p in group_pages)
    block_table = torch.zeros(len(group_pages), width, dtype=torch.int32,
                              device="cpu" if on_host else device)
    for g, p in enumerate(group_pages):
        block_table[g, : p.numel()] = p
    if on_host:  # one upload instead of one copy per request
        block_table = block_table.pin_memory().to(device, non_blocking=True)
    lens_host = torch.tensor([enc_lens[i] for i in firsts], dtype=torch.int32)
    qsl_host = torch.tensor(offsets, dtype=torch.int32)
    metadata = paged_ops.get_scheduler_metadata(
        num_reqs=len(group_pages), num_heads=attn.num_heads, num_kv_heads=attn.num_heads,
        head_dim=attn.head_dim, seq_lens=lens_host, dtype=attn.k_cache.dtype,
        query_start_loc=qsl_host, causal=False, isa=isa, block_size=block_size)
    seq_lens = lens_host.to(device, non_blocking=True)
    qsl = qsl_host.to(device, non_blocking=True)
    return [(layer.encoder_attn.k_cache, layer.encoder_attn.v_cache, block_table, seq_lens, metadata, qsl)
            for layer in layers]


@torch.library.custom_op("vflorence::self_attention", mutates_args={"k_cache", "v_cache"})
def decoder_self_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                           k_cache: torch.Tensor, v_cache: torch.Tensor, scale: float) -> torch.Tensor:
    """Write this step's K/V into the paged cache, then attend over each sequence's cache - in
    one launch where the plan allows it (the attention kernel stores each row's new K/V ahead of
    reading the block that holds it), else the append kernel and then the attention."""
    ctx = get_context()
    out = torch.empty_like(query)
    # causal=False is still causal: each sequence queries only its newest token, and the cache
    # holds nothing after it.
    if ctx.self_groups is not None:  # the beams of a request share one CTA, each row its own table
        qsl, lens = ctx.self_groups, ctx.self_group_lens
    else:
        qsl, lens = ctx.query_start_loc, ctx.context_lens
    if ctx.self_append is None:
        ctx.self_append = paged_ops.attention_append_supported(ctx.self_metadata)
    if ctx.self_append:
        paged_ops.attention_with_kv_cache_append(query, key, value, k_cache, v_cache, out, ctx.slot_mapping, qsl,
                                                 lens, scale=scale, causal=False, block_table=ctx.block_tables,
                                                 scheduler_metadata=ctx.self_metadata)
        return out
    paged_ops.reshape_and_cache(key, value, k_cache, v_cache, ctx.slot_mapping, isa=ctx.isa)
    paged_ops.attention_with_kv_cache(query, k_cache, v_cache, out, qsl, lens, scale=scale, causal=False,
                                      block_table=ctx.block_tables, scheduler_metadata=ctx.self_metadata)
    return out


@decoder_self_attention.register_fake
def _(query, key, value, k_cache, v_cache, scale):
    return torch.empty_like(query)


@torch.library.custom_op("vflorence::cross_attention", mutates_args={})
def decoder_cross_attention(query: torch.Tensor, layer_idx: int, scale: float) -> torch.Tensor:
    """Cross-attention of decoder layer ``layer_idx`` over the staged encoder K/V pages. Takes this
    module's staging (6-tuples with the beams' grouped ``query_start_loc``) or the reference's
    (5-tuples, one request per row, with the Context's ``query_start_loc``,
    vflorence/layers/attention.py:97-109)."""
    ctx = get_context()
    staged = ctx.cross_staged[layer_idx]
    if len(staged) == 5:
        (k_cache, v_cache, block_table, seq_lens, metadata), qsl = staged, ctx.query_start_loc
    else:
        k_cache, v_cache, block_table, seq_lens, metadata, qsl = staged
    out = torch.empty_like(query)
    paged_ops.attention_with_kv_cache(query, k_cache, v_cache, out, qsl, seq_lens, scale=scale,
                                      causal=False, block_table=block_table, scheduler_metadata=metadata)
    return out


@decoder_cross_attention.register_fake
def _(query, layer_idx, scale):
    return torch.empty_like(query)
