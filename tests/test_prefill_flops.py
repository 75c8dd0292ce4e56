"""The prefill roofline's numerator (bench.prefill_flops) on the 8B shape.

The prompt path's algorithmic work is the full-model count (2 FLOPs per weight
per token for every decoder matrix, plus 4 * heads * head_dim per causal
query-key pair and layer for q.k and p.v) minus what a prompt never needs: the
last layer's output projection, FFN and attention (only its K/V append
matters) and the LM head.
"""
from __future__ import annotations

import types

import bench
from dotnetfoundryllm_b200 import ggufgen


def _desc(name: str):
    s = ggufgen.SPECS[name]
    return types.SimpleNamespace(n_heads=s.n_heads, head_dim=s.hd, n_kv_heads=s.n_kv, hidden=s.hidden, ffn=s.ffn,
                                 n_layers=s.n_layers)


def test_prefill_flops_8b():
    d = _desc("llama3-8b")
    n = 2047
    qd, kvd, h, f, L = d.n_heads * d.head_dim, d.n_kv_heads * d.head_dim, d.hidden, d.ffn, d.n_layers
    per_layer = h * (qd + 2 * kvd) + qd * h + 3 * h * f
    assert L * per_layer == 6_979_321_856  # decoder weights of the 8B shape
    pairs = n * (n + 1) // 2
    full = 2 * n * L * per_layer + 4 * d.n_heads * d.head_dim * pairs * L
    skipped = 2 * n * (qd * h + 3 * h * f) + 4 * d.n_heads * d.head_dim * pairs
    assert bench.prefill_flops(d, n) == full - skipped == 28_848_087_367_680
