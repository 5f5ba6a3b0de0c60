"""ORACLE — test infrastructure only.

A stand-in for the external ``vllm_cpu_attn`` package (not installable here) with the four
functions the vflorence engine calls, backed by the C restatement in ``oracle/paged_ref.c``.
It is put on ``sys.path`` only by ``tests/golden/make_golden.py`` so that the unmodified
reference engine can run on this machine and record golden traces.

Call sites it serves (paths inside the vflorence project): get_isa
(vflorence/engine/model_runner.py:38), get_scheduler_metadata (vflorence/layers/attention.py:18,
model_runner.py:308), reshape_and_cache (attention.py:55, model_runner.py:252),
attention_with_kv_cache (attention.py:61, :98).
"""

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import oracle as _oracle  # noqa: E402

# Every call is recorded here when RECORD is a list (used by the golden-trace generator).
RECORD = None


def get_isa(dtype, block_size, head_dim):
    return "oracle"


def get_scheduler_metadata(num_reqs, num_heads, num_kv_heads, head_dim, seq_lens, dtype,
                           query_start_loc, causal, isa, block_size):
    # The CPU kernel's work partition has no observable effect on results.
    return torch.empty(0, dtype=torch.int32)


def reshape_and_cache(key, value, k_cache, v_cache, slot_mapping, isa=None):
    if RECORD is not None:
        RECORD.append(("reshape_and_cache", slot_mapping.clone(), key.shape[0]))
    bad = _oracle.reshape_and_cache(key, value, k_cache, v_cache, slot_mapping)
    if bad:
        raise RuntimeError(f"oracle: {bad} out-of-range slots")


def attention_with_kv_cache(query, k_cache, v_cache, output, query_start_loc, seq_lens, scale,
                            causal, block_table, scheduler_metadata):
    bad = _oracle.attention(query, k_cache, v_cache, output, query_start_loc, seq_lens, scale,
                            causal, block_table)
    if bad:
        raise RuntimeError(f"oracle: {bad} rows with out-of-range block ids")
