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


@pytest.mark.parametrize("m,n,k,ks", [(128, 64, 8192, 4), (4096, 64, 2 * 14336, 10), (300, 130, 1000, 3)])
def test_k_split_matches_fp32_product(m, n, k, ks):
    """Skinny products (the batched steps) split their K range over several
    work items; the partials are summed in split order (deterministic)."""
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float16)
    b = rng.standard_normal((n, k)).astype(np.float16)
    y0 = rng.standard_normal((1, n, m)).astype(np.float32)
    got = runtime.gemm_f16(a, b, m, n, k, alpha=0.25, beta=1.0, y=y0, ksplit=ks)
    _check(got, a, b, m, n, k, 0.25, 1.0, y0[0])
    again = runtime.gemm_f16(a, b, m, n, k, alpha=0.25, beta=1.0, y=y0, ksplit=ks)
    np.testing.assert_array_equal(got, again)


def test_causal_modes():
    """The prompt path's attention: mode 1 leaves scores of keys past a row's
    causal bound (per 128-key x token tile) unwritten and every needed score
    exact; mode 2 cuts each of 3 K segments to the bound, exact where the
    operand past it is zero (the softmax's probabilities are)."""
    rng = np.random.default_rng(11)
    grp, start, ntok, hd = 4, 100, 300, 128
    nk = start + ntok
    nkp = (nk + 63) // 64 * 64
    rows = ntok * grp
    keys = rng.standard_normal((nkp, 3 * hd)).astype(np.float16)
    q = rng.standard_normal((rows, 3 * hd)).astype(np.float16)
    sentinel = np.full((1, rows, nkp), 7.0, np.float32)
    got = runtime.gemm_f16(keys, q, nkp, rows, 3 * hd, y=sentinel, causal=1, c_grp=grp, c_start=start)[0]
    ref = q.astype(np.float32) @ keys.astype(np.float32).T
    for r in range(0, rows, 37):
        kb = start + r // grp + 1  # keys a row may see
        np.testing.assert_allclose(got[r, :kb], ref[r, :kb], rtol=1e-5, atol=1e-3)
    # probabilities zero past each row's keys, three segments of nkp
    p = rng.random((rows, nkp)).astype(np.float32)
    for r in range(rows):
        p[r, start + r // grp + 1:] = 0.0
    p16 = p.astype(np.float16)
    P = np.concatenate([p16, p16, p16], 1)
    vt = rng.standard_normal((hd, 3 * nkp)).astype(np.float16)
    got2 = runtime.gemm_f16(vt, P, hd, rows, 3 * nkp, causal=2, c_grp=grp, c_start=start, c_seg=3)[0]
    ref2 = P.astype(np.float32) @ vt.astype(np.float32).T
    np.testing.assert_allclose(got2, ref2, rtol=1e-4, atol=1e-3)
