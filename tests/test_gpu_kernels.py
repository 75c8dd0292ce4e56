"""Kernel-level parity on the GPU, through the C ABI.

- ``fl_dequant``: the device dequantizer is bit-exact against the reference
  decoder (oracle) for every supported type, on generator blocks and on raw
  random bytes (NaN payloads exact for the F32/F16/BF16 conversions,
  compared by class where a NaN scale goes through the block arithmetic), and on the reference's own
  known-answer blocks.
- ``fl_matvec``: the fused dequant-matvec kernel (repack + int8 tensor-core
  MMA + scale epilogue) against LinearProjection over the oracle's F32 weights,
  for every quantized format, aligned and straddling rows, and full Llama-3-8B
  projection shapes.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from dotnetfoundryllm_b200 import ggufgen, runtime
from dotnetfoundryllm_b200.gguf import BLOCK, T_Q4_0, T_Q4_K, T_Q5_K, T_Q6_K, T_Q8_0, T_Q8_K, TYPE_NAMES
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ALL_TYPES = [0, 1, 2, 8, 12, 13, 14, 15, 30]
KQ = (T_Q4_K, T_Q5_K, T_Q6_K, T_Q8_K)
KATS = json.loads((Path(__file__).parent / "golden" / "reference_kats.json").read_text())


# Conversions without arithmetic: every bit, NaN payloads included (a half
# NaN comes back quiet with its payload, as (float)Half does).
EXACT_NAN = (0, 1, 30)


def _bits_equal(a: np.ndarray, b: np.ndarray, t: int) -> None:
    """Bit equality.  For the block formats a NaN scale propagates through the
    products; which NaN an x86 multiply returns depends on the operand order
    the host compiler picked and the GPU returns the canonical NaN, so there
    NaNs are compared by class; every other value bit for bit."""
    if t in EXACT_NAN:
        ia, ib = a.view(np.uint32), b.view(np.uint32)
        bad = np.nonzero(ia != ib)[0]
        assert bad.size == 0, f"{bad.size} values differ, first at {bad[0]}: {ia[bad[0]]:#x} vs {ib[bad[0]]:#x}"
        return
    na, nb = np.isnan(a), np.isnan(b)
    assert (na == nb).all(), "NaN class differs"
    ia, ib = a[~na].view(np.uint32), b[~nb].view(np.uint32)
    bad = np.nonzero(ia != ib)[0]
    assert bad.size == 0, f"{bad.size} values differ, first at {bad[0]}: {a[~na][bad[0]]} vs {b[~nb][bad[0]]}"


@pytest.mark.parametrize("t", ALL_TYPES, ids=lambda t: TYPE_NAMES.get(t, str(t)))
def test_dequant_bit_exact_generated(t):
    raw = ggufgen.random_blocks(t, 256 * 64, 21, 500 + t)
    rc, ref = O.dequantize(t, raw)
    assert rc == O.OK
    _bits_equal(runtime.dequantize(t, raw), ref, t)


@pytest.mark.parametrize("t", ALL_TYPES, ids=lambda t: TYPE_NAMES.get(t, str(t)))
def test_dequant_bit_exact_random_bytes(t):
    be, bb = BLOCK[t]
    rng = np.random.default_rng(1234 + t)
    raw = rng.integers(0, 256, size=bb * (4096 // be if be > 1 else 4096), dtype=np.uint8)
    rc, ref = O.dequantize(t, raw)
    assert rc == O.OK
    _bits_equal(runtime.dequantize(t, raw), ref, t)


@pytest.mark.parametrize("e", KATS["dequantize"], ids=lambda e: e["name"])
def test_dequant_reference_known_blocks(e):
    raw = np.frombuffer(bytes.fromhex(e["hex"]), dtype=np.uint8)
    out = runtime.dequantize(e["type"], raw)
    if "expect_all" in e:
        np.testing.assert_array_equal(out, np.array(e["expect_all"], dtype=np.float32))
    for k, v in e.get("expect", {}).items():
        assert out[int(k)] == np.float32(v)


def test_dequant_empty_and_errors():
    assert runtime.dequantize(12, np.zeros(0, np.uint8)).size == 0
    with pytest.raises(runtime.NotSupportedError):
        runtime.dequantize(99, np.zeros(4, np.uint8), 1)
    with pytest.raises(runtime.ArgumentError):
        runtime.dequantize(12, np.zeros(143, np.uint8), 256)


MV_SHAPES = [(48, 512), (32, 1408), (40, 256), (24, 1024), (160, 4096)]


@pytest.mark.parametrize("t", [T_Q4_K, T_Q5_K, T_Q6_K, T_Q8_0, T_Q4_0, T_Q8_K], ids=lambda t: TYPE_NAMES[t])
@pytest.mark.parametrize("shape", MV_SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_matvec_matches_oracle(t, shape):
    rows, cols = shape
    if (rows * cols) % (256 if t in KQ else 32):
        pytest.skip("not whole blocks")
    raw = ggufgen.random_blocks(t, rows * cols, 31, 900 + t)
    x = ggufgen.normal(cols, 32, 5)
    y_ref = O.matvec(t, raw, rows, cols, x)
    y = runtime.matvec(t, raw, rows, cols, x)
    np.testing.assert_allclose(y, y_ref, rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("t,rows,cols", [(T_Q4_K, 4096, 4096), (T_Q6_K, 4096, 14336), (T_Q5_K, 3584, 4096),
                                         (T_Q8_0, 1024, 4096)], ids=["8b-wq", "8b-down", "g9b-wo", "m7b-wk"])
def test_matvec_full_size_shapes(t, rows, cols):
    raw = ggufgen.random_blocks(t, rows * cols, 41, 77)
    x = ggufgen.normal(cols, 42, 6)
    y_ref = O.matvec(t, raw, rows, cols, x)
    y = runtime.matvec(t, raw, rows, cols, x)
    np.testing.assert_allclose(y, y_ref, rtol=1e-4, atol=5e-5)


def test_matvec_zero_input():
    raw = ggufgen.random_blocks(T_Q4_K, 64 * 512, 1, 1)
    x = np.zeros(512, np.float32)
    y = runtime.matvec(T_Q4_K, raw, 64, 512, x)
    np.testing.assert_array_equal(y, np.zeros(64, np.float32))
