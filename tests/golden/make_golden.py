"""Generate the golden fixtures under tests/golden/ (run once, on a machine with the reference).

    python tests/golden/make_golden.py --reference-root <path to the vflorence checkout>

Two fixture sets:

1. ``attention_cases.npz`` — paged attention cases with the expected output computed by torch
   in float64 on a dense gather of the pages (independent of the C oracle). Pins the oracle's
   attention arithmetic and serves as a fixed GPU parity target.

2. ``engine_trace.pt`` — the UNMODIFIED reference engine (vflorence, block_size 16, fp32,
   ``compile=False``) run on a small random BART with ``oracle/vllm_cpu_attn`` standing in for the
   un-installable ``vllm_cpu_attn`` package. Recorded per decode step: the Context tensors built
   by ``ModelRunner._prepare`` (vflorence/engine/model_runner.py:273-341), the copy-on-write pairs
   (model_runner.py:162-167), the cross-attention staging (vflorence/layers/attention.py:9-39),
   encoder slots (model_runner.py:232-259), the log of BlockManager calls
   (vflorence/engine/block_manager.py) and final token ids; plus HuggingFace transformers'
   ``generate`` tokens for the same requests (asserted equal: this pins the oracle end to end),
   and snapshots of a few attention calls (inputs, pool contents, output).

The reference is imported from ``--reference-root`` only by this script; tests read the
committed fixtures.
"""

from __future__ import annotations

import argparse
import math
import os
import sys
import weakref
from tempfile import TemporaryDirectory

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


# --------------------------------------------------------------------------------------------
# 1. attention cases (float64 expectation; no reference import needed)
# --------------------------------------------------------------------------------------------

def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def _expected(q, kc, vc, qsl, lens, table, scale, causal):
    """float64 softmax attention over a dense gather of each request's pages."""
    q, kc, vc = q.double(), kc.double(), vc.double()
    bs = kc.shape[2]
    out = torch.zeros_like(q)
    for r in range(len(lens)):
        n = int(lens[r])
        q0, q1 = int(qsl[r]), int(qsl[r + 1])
        if n <= 0:
            continue
        blocks = [int(table[r, t // bs]) for t in range(n)]
        offs = [t % bs for t in range(n)]
        K = kc[blocks, :, offs]  # [n, H, D]
        V = vc[blocks, :, offs]
        for i in range(q0, q1):
            vis = n - (q1 - 1 - i) if causal else n
            if vis <= 0:
                continue
            s = torch.einsum("hd,thd->ht", q[i], K[:vis]) * scale
            p = torch.softmax(s, dim=-1)
            out[i] = torch.einsum("ht,thd->hd", p, V[:vis])
    return out


def attention_cases(seed: int = 7):
    g = torch.Generator().manual_seed(seed)
    cases = []

    def make(name, *, heads, head_dim, block_size, lens, q_lens=None, causal=False,
             num_blocks=None, dtype="f32", table_cols=None):
        nreq = len(lens)
        q_lens = q_lens or [1] * nreq
        need = [max(1, math.ceil(n / block_size)) for n in lens]
        cols = table_cols or max(need)
        nb = num_blocks or (sum(need) + 3)
        perm = torch.randperm(nb, generator=g)
        table = torch.zeros(nreq, cols, dtype=torch.int32)
        pos = 0
        for r, k in enumerate(need):
            table[r, :k] = perm[pos:pos + k].to(torch.int32)
            pos += k
        # bf16-representable inputs so the same bytes serve fp32 and bf16 kernels
        kc = torch.randn(nb, heads, block_size, head_dim, generator=g).to(torch.bfloat16)
        vc = torch.randn(nb, heads, block_size, head_dim, generator=g).to(torch.bfloat16)
        total_q = sum(q_lens)
        q = torch.randn(total_q, heads, head_dim, generator=g).to(torch.bfloat16)
        qsl = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.int32)
        lens_t = torch.tensor(lens, dtype=torch.int32)
        scale = head_dim ** -0.5
        exp = _expected(q.float(), kc.float(), vc.float(), qsl, lens_t, table, scale, causal)
        cases.append(dict(name=name, dtype=dtype, causal=int(causal), scale=scale,
                          block_size=block_size, q=_bf16_bits(q), k_cache=_bf16_bits(kc),
                          v_cache=_bf16_bits(vc), query_start_loc=qsl.numpy(),
                          seq_lens=lens_t.numpy(), block_table=table.numpy(),
                          expected=exp.numpy()))

    # one query per sequence (decoder self-attention), ragged lengths around block edges
    make("self_edges_f32", heads=2, head_dim=64, block_size=16,
         lens=[1, 15, 16, 17, 31, 32, 33, 48])
    make("self_edges_bf16", heads=2, head_dim=64, block_size=16, dtype="bf16",
         lens=[1, 15, 16, 17, 31, 32, 33, 48])
    make("self_long_bf16", heads=2, head_dim=64, block_size=16, dtype="bf16", lens=[400, 93, 257])
    make("self_bs32_f32", heads=2, head_dim=64, block_size=32, lens=[1, 31, 32, 33, 100])
    make("self_d128_bf16", heads=2, head_dim=128, block_size=16, dtype="bf16", lens=[5, 40, 77])
    make("self_d32_f32", heads=3, head_dim=32, block_size=16, lens=[9, 64, 65])
    # beams sharing one encoder: several query rows per request, non-causal (cross-attention)
    make("cross_beams_bf16", heads=2, head_dim=64, block_size=16, dtype="bf16",
         lens=[577, 200, 33], q_lens=[3, 4, 1])
    make("cross_beams_f32", heads=2, head_dim=64, block_size=16, lens=[64, 17], q_lens=[5, 2])
    # causal multi-query rows and a request with nothing visible
    make("causal_f32", heads=2, head_dim=64, block_size=16, lens=[20, 3, 0], q_lens=[4, 3, 1],
         causal=True)
    # empty context (zero output) next to normal rows; wider table than needed
    make("zero_len_bf16", heads=2, head_dim=64, block_size=16, dtype="bf16", lens=[0, 12, 0, 40],
         table_cols=6)
    return cases


def save_attention_cases(path):
    cases = attention_cases()
    flat = {}
    for i, c in enumerate(cases):
        for k, v in c.items():
            flat[f"{i}:{k}"] = np.asarray(v)
    flat["num_cases"] = np.asarray(len(cases))
    np.savez_compressed(path, **flat)
    print(f"wrote {path}: {len(cases)} cases, {os.path.getsize(path)} bytes")


# --------------------------------------------------------------------------------------------
# 2. reference engine trace
# --------------------------------------------------------------------------------------------

def engine_trace(reference_root: str, out_path: str):
    sys.path.insert(0, os.path.join(REPO, "oracle"))  # vllm_cpu_attn stand-in
    sys.path.insert(0, reference_root)
    import vllm_cpu_attn  # noqa: F401  (the oracle stand-in)
    import vflorence.config as vconfig

    vconfig.AARCH64 = True  # block_size 16, the BASELINE block size (only affects compile choices otherwise)
    from transformers import BartConfig
    from transformers import BartForConditionalGeneration as HFBart

    import vflorence.engine.model_runner as mr
    from vflorence import LLM, Request, SamplingParams
    from vflorence.engine.block_manager import BlockManager

    torch.manual_seed(0)
    cfg = BartConfig(vocab_size=96, d_model=128, encoder_layers=2, decoder_layers=2,
                     encoder_attention_heads=2, decoder_attention_heads=2, encoder_ffn_dim=256,
                     decoder_ffn_dim=256, max_position_embeddings=160, decoder_start_token_id=1,
                     eos_token_id=2, pad_token_id=0, bos_token_id=0, forced_eos_token_id=None,
                     init_std=0.2)
    hf = HFBart(cfg).eval()

    # ---- recording hooks (wrap, never modify, the reference) ----
    uid = weakref.WeakKeyDictionary()
    counter = [0]

    def seq_id(seq):
        # monotonic ids: live sequences never share one, even after others are collected
        if seq not in uid:
            uid[seq] = counter[0]
            counter[0] += 1
        return uid[seq]

    trace = {"runs": []}
    cur = {}

    orig = {name: getattr(BlockManager, name) for name in
            ("ensure_capacity", "fork", "deallocate", "required_new_blocks", "reset")}

    def rec(op):
        cur["bm_log"].append(op)

    def ensure_capacity(self, seq):
        before = list(seq.block_table)
        res = orig["ensure_capacity"](self, seq)
        rec(("ensure", seq_id(seq), seq.num_cached_tokens, before,
             None if res is None else tuple(res), list(seq.block_table)))
        return res

    def fork(self, parent, child):
        orig["fork"](self, parent, child)
        rec(("fork", seq_id(parent), seq_id(child), list(child.block_table)))

    def deallocate(self, seq):
        table = list(seq.block_table)
        orig["deallocate"](self, seq)
        rec(("dealloc", seq_id(seq), table, list(self.free_block_ids)))

    def required_new_blocks(self, seqs):
        res = orig["required_new_blocks"](self, seqs)
        rec(("required", [seq_id(s) for s in seqs], res))
        return res

    def reset(self):
        orig["reset"](self)
        if "bm_log" in cur:
            rec(("reset",))

    BlockManager.ensure_capacity = ensure_capacity
    BlockManager.fork = fork
    BlockManager.deallocate = deallocate
    BlockManager.required_new_blocks = required_new_blocks
    BlockManager.reset = reset

    orig_prepare = mr.ModelRunner._prepare
    orig_copy = mr.ModelRunner._copy_blocks
    orig_set_context = mr.set_context
    orig_encode = mr.ModelRunner._encode

    def _prepare(self, seqs, copies=()):
        step = {"seqs": [seq_id(s) for s in seqs],
                "request_ids": [s.request_id for s in seqs],
                "positions": [s.num_cached_tokens for s in seqs],
                "block_tables": [list(s.block_table) for s in seqs],
                "copies": [tuple(c) for c in copies]}
        cur["steps"].append(step)
        return orig_prepare(self, seqs, copies)

    def _copy_blocks(self, copies):
        cur["steps"][-1]["copies_applied"] = [tuple(c) for c in copies]
        return orig_copy(self, copies)

    def set_context(**fields):
        if fields:
            step = cur["steps"][-1]
            for k in ("context_lens", "block_tables", "slot_mapping", "query_start_loc"):
                step["ctx_" + k] = fields[k].clone()
            kc, vc, table, lens, _ = fields["cross_staged"][0]
            step["cross_block_table"] = table.clone()
            step["cross_seq_lens"] = lens.clone()
        return orig_set_context(**fields)

    def _encode(self, seqs):
        # same grouping as the reference (model_runner.py:215-220): by encoder length (text only)
        groups = {}
        for s in seqs:
            groups.setdefault(len(s.encoder_token_ids), []).append(s.request_id)
        free_before = list(self._cross_free)
        vllm_cpu_attn.RECORD = []
        orig_encode(self, seqs)
        calls = vllm_cpu_attn.RECORD
        vllm_cpu_attn.RECORD = None
        L = len(self.decoder_layers)
        cur["encodes"].append({
            "seqs": [seq_id(s) for s in seqs],
            "request_ids": [s.request_id for s in seqs],
            "enc_lens": [len(s.encoder_token_ids) for s in seqs],
            "groups": [(rids, n) for n, rids in groups.items()],
            "group_slots": [calls[g * L][1] for g in range(len(groups))],
            "cross_pages": {rid: (p.clone(), n) for rid, (p, n) in self._cross_pages.items()},
            "cross_free_before": free_before,
            "cross_free_after": list(self._cross_free),
        })

    orig_clear = mr.ModelRunner.clear_request

    def clear_request(self, request_id):
        orig_clear(self, request_id)
        cur["clears"].append((request_id, list(self._cross_free)))

    mr.ModelRunner.clear_request = clear_request
    mr.ModelRunner._prepare = _prepare
    mr.ModelRunner._copy_blocks = _copy_blocks
    mr.set_context = set_context
    mr.ModelRunner._encode = _encode

    # attention snapshots: wrap the stand-in's attention to capture a few calls
    snap = {"want": set(), "calls": 0, "out": []}
    orig_attn = vllm_cpu_attn.attention_with_kv_cache

    def attention_with_kv_cache(query, k_cache, v_cache, output, query_start_loc, seq_lens,
                                scale, causal, block_table, scheduler_metadata):
        orig_attn(query, k_cache, v_cache, output, query_start_loc, seq_lens, scale, causal,
                  block_table, scheduler_metadata)
        snap["calls"] += 1
        if snap["calls"] in snap["want"]:
            snap["out"].append({"query": query.clone(), "k_cache": k_cache.clone(),
                                "v_cache": v_cache.clone(), "output": output.clone(),
                                "query_start_loc": query_start_loc.clone(),
                                "seq_lens": seq_lens.clone(), "block_table": block_table.clone(),
                                "scale": scale, "causal": causal, "call": snap["calls"]})

    vllm_cpu_attn.attention_with_kv_cache = attention_with_kv_cache

    rng = np.random.default_rng(11)
    workloads = [
        dict(name="greedy", max_num_seqs=3, max_decoder_len=48,
             params=dict(max_tokens=40, min_length=41), enc_lens=[5, 23, 40, 17],
             snapshot_calls={149, 150}),
        dict(name="beam2", max_num_seqs=4, max_decoder_len=32,
             params=dict(max_tokens=20, num_beams=2, length_penalty=2.0, no_repeat_ngram_size=3),
             enc_lens=[12, 30, 7], snapshot_calls={61, 62}),
        dict(name="beam4", max_num_seqs=8, max_decoder_len=48,
             params=dict(max_tokens=36, num_beams=4, min_length=37), enc_lens=[9, 26],
             snapshot_calls={101, 102}),
    ]
    with TemporaryDirectory() as path:
        hf.save_pretrained(path)
        for w in workloads:
            cur.clear()
            cur.update(steps=[], encodes=[], bm_log=[], clears=[])
            snap.update(want=w["snapshot_calls"], calls=0, out=[])
            reqs = [rng.integers(3, cfg.vocab_size, size=n).tolist() for n in w["enc_lens"]]
            llm = LLM(path, max_num_seqs=w["max_num_seqs"], compile=False,
                      max_decoder_len=w["max_decoder_len"])
            assert llm.config.block_size == 16
            params = SamplingParams(**w["params"])
            effective = params.with_defaults(llm._sampling_params)
            outs = llm.generate([Request(r) for r in reqs], params, use_tqdm=False)
            tokens = [o.completion_token_ids for o in outs]
            hf_tokens = []
            for r in reqs:
                kw = dict(max_new_tokens=w["params"]["max_tokens"],
                          num_beams=w["params"].get("num_beams", 1), do_sample=False)
                for k in ("min_length", "length_penalty", "no_repeat_ngram_size"):
                    if k in w["params"]:
                        kw[k] = w["params"][k]
                with torch.no_grad():
                    ref = hf.generate(torch.tensor([r]), **kw)
                hf_tokens.append(ref[0].tolist()[1:])
            match = [a == b[: len(a)] and len(a) == len(b) for a, b in zip(tokens, hf_tokens)]
            print(f"{w['name']}: {len(cur['steps'])} steps, "
                  f"{sum(len(s['copies']) for s in cur['steps'])} CoW pairs, "
                  f"tokens == HF generate: {match}")
            assert all(match), (tokens, hf_tokens)
            trace["runs"].append({
                "name": w["name"], "config": {k: v for k, v in w.items() if k != "snapshot_calls"},
                "sampling": {f: getattr(effective, f) for f in effective.__slots__},
                "model_config": cfg.to_dict(),
                "decoder_start_token_id": cfg.decoder_start_token_id,
                "block_size": llm.config.block_size, "num_blocks": llm.config.num_blocks,
                "num_cross_blocks": llm.config.num_cross_blocks,
                "num_heads": 2, "head_dim": 64, "num_layers": cfg.decoder_layers,
                "requests": reqs, "tokens": tokens, "hf_tokens": hf_tokens,
                "steps": cur["steps"], "encodes": cur["encodes"], "bm_log": cur["bm_log"],
                "clears": cur["clears"],
                "attention_snapshots": snap["out"],
            })
    trace["model_state"] = {k: v.clone() for k, v in hf.state_dict().items()}
    torch.save(trace, out_path)
    print(f"wrote {out_path}: {os.path.getsize(out_path)} bytes")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", required=False,
                    help="vflorence checkout (needed for engine_trace.pt)")
    ap.add_argument("--only", choices=["attention", "engine"], default=None)
    args = ap.parse_args()
    if args.only in (None, "attention"):
        save_attention_cases(os.path.join(HERE, "attention_cases.npz"))
    if args.only in (None, "engine"):
        if not args.reference_root:
            ap.error("--reference-root is required for the engine trace")
        engine_trace(args.reference_root, os.path.join(HERE, "engine_trace.pt"))


if __name__ == "__main__":
    main()
