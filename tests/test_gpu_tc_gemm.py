"""The tcgen05 GEMM of the prompt path and of batched decode (fl_gemm_f16
test hook, the kernel behind fl_prefill and fl_forward_batch) against a plain
fp32 product of the same fp16 operands.

fp16 operands are exact in fp32, so the only difference is the order of the
fp32 accumulation: |got - ref| <= 1e-5 * sum_k |a_k b_k| + 1e-6 bounds it.
Shapes cover one tile, ragged edges on every axis (TMA zero fill past the
matrix, masked stores), each token-tile width (64, 128, 256), long K (the
split-fp16 3K of a 14336-wide input), several tiles per CTA of the persistent
grid, batches with padded rows between them (attention's per-kv-head
products) and the beta = 1 accumulation of the batched steps.
"""
from __future__ import annotations

import numpy as np
import pytest

from dotnetfoundryllm_b200 import runtime

pytestmark = pytest.mark.gpu


def _check(got, a, b, m, n, k, alpha, beta=0.0, y0=None):
    af = a[..., :m, :k].astype(np.float32)
    bf = b[..., :n, :k].astype(np.float32)
    ref = alpha * np.einsum("...mk,...nk->...nm", af, bf)
    mag = abs(alpha) * np.einsum("...mk,...nk->...nm", np.abs(af), np.abs(bf))
    if y0 is not None:
        ref = ref + beta * y0
        mag = mag + abs(beta) * np.abs(y0)
    err = np.abs(got.reshape(ref.shape) - ref)
    bound = 1e-5 * mag + 1e-6
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), f"at {worst}: {got.reshape(ref.shape)[worst]} vs {ref[worst]}"


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (200, 300, 136), (128, 40, 64), (384, 100, 512),
                                   (1000, 130, 1000), (256, 2048, 3 * 4096), (130, 17, 3 * 14336),
                                   (4096, 256, 256)])
def test_matches_fp32_product(m, n, k):
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    ld = (k + 7) // 8 * 8 + 8  # row stride wider than k: columns past k are never read
    a = rng.standard_normal((m, ld)).astype(np.float16)
    b = rng.standard_normal((n, ld)).astype(np.float16)
    got = runtime.gemm_f16(a, b, m, n, k, alpha=0.5)
    _check(got, a, b, m, n, k, 0.5)


def test_batched_with_padded_rows():
    rng = np.random.default_rng(5)
    batch, m, n, k, ra, rb = 3, 100, 72, 384, 104, 80
    a = rng.standard_normal((batch, ra, k)).astype(np.float16)
    b = rng.standard_normal((batch, rb, k)).astype(np.float16)
    got = runtime.gemm_f16(a, b, m, n, k, batch=batch, a_batch_rows=ra, b_batch_rows=rb)
    _check(got, a, b, m, n, k, 1.0)


def test_beta_accumulates_into_y():
    rng = np.random.default_rng(6)
    m, n, k = 300, 64, 4096
    a = rng.standard_normal((m, k)).astype(np.float16)
    b = rng.standard_normal((n, k)).astype(np.float16)
    y0 = rng.standard_normal((1, n, m)).astype(np.float32)
    got = runtime.gemm_f16(a, b, m, n, k, alpha=1.0 / 256, beta=1.0, y=y0)
    _check(got, a, b, m, n, k, 1.0 / 256, 1.0, y0[0])
