"""CPU checks of the device weight layout and the matvec arithmetic.

``fl_repack`` turns raw GGUF blocks into the unit layout the kernel streams;
``fl_emulate_matvec`` reads that layout exactly the way the kernel does
(fragment registers, scale pairs, 3-limb int8 input) and forms the same
integer sums.  Comparing it with the oracle's F32 LinearProjection pins the
layout and the arithmetic without a GPU.  The generator is checked for
determinism and for producing blocks the reference decoder maps back to the
sampled values."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from dotnetfoundryllm_b200 import _native as N
from dotnetfoundryllm_b200 import ggufgen
from dotnetfoundryllm_b200.gguf import T_Q4_0, T_Q4_K, T_Q5_K, T_Q6_K, T_Q8_0, T_Q8_K, TYPE_NAMES
from oracle import oracle as O

KQ = (T_Q4_K, T_Q5_K, T_Q6_K, T_Q8_K)
TYPES = [T_Q4_K, T_Q5_K, T_Q6_K, T_Q8_0, T_Q4_0, T_Q8_K]
# (rows, cols): aligned, straddling rows (1408 = 5.5 super-blocks, the tiny
# config's ffn_down), a single k-block, rows not a multiple of 16
SHAPES = [(48, 512), (32, 1408), (40, 256), (24, 1024)]


def _layout(t, rows, cols):
    L = N.FlMatrixLayout()
    assert N.cuda().fl_layout_for(t, rows, cols, C.byref(L)) == 0
    return L


def _emulate(t, raw, rows, cols, x):
    L = _layout(t, rows, cols)
    packed = np.zeros(L.total_bytes, np.uint8)
    N.cuda().fl_repack(C.byref(L), raw.ctypes.data_as(C.c_void_p), None, None, packed.ctypes.data_as(C.c_void_p), 0)
    y = np.zeros(rows, np.float32)
    N.cuda().fl_emulate_matvec(C.byref(L), packed.ctypes.data_as(C.c_void_p), x.ctypes.data_as(C.c_void_p),
                               y.ctypes.data_as(C.c_void_p))
    return y, L


@pytest.mark.parametrize("t", TYPES, ids=lambda t: TYPE_NAMES[t])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_emulated_kernel_matches_oracle(t, shape):
    rows, cols = shape
    if (rows * cols) % (256 if t in KQ else 32):
        pytest.skip("element count not a whole number of blocks")
    raw = ggufgen.random_blocks(t, rows * cols, 11, 1000 + t)
    x = ggufgen.normal(cols, 12, 77)
    y_ref = O.matvec(t, raw, rows, cols, x)
    y, L = _emulate(t, raw, rows, cols, x)
    assert L.expanded == (1 if (t in KQ and cols % 256) else 0)
    np.testing.assert_allclose(y, y_ref, rtol=1e-4, atol=2e-5)


def test_unit_sizes_equal_gguf_blocks():
    """A unit carries exactly the bytes of 16 GGUF blocks (Q8_K drops bsums)."""
    expect = {T_Q4_K: 16 * 144, T_Q5_K: 16 * 176, T_Q6_K: 16 * 210, T_Q8_0: 16 * 8 * 34, T_Q4_0: 16 * 8 * 18,
              T_Q8_K: 16 * 260}
    for t, b in expect.items():
        assert _layout(t, 16, 256).unit_bytes == b
        assert _layout(t, 16, 256).total_bytes == b


def test_layout_rejects_ragged_rows():
    L = N.FlMatrixLayout()
    assert N.cuda().fl_layout_for(T_Q4_K, 16, 48, C.byref(L)) == -2
    assert N.cuda().fl_layout_for(0, 16, 256, C.byref(L)) == -1


def test_interleaved_gate_up_repack():
    """The gate/up interleave (tile rows 0..7 gate, 8..15 up) reproduces both
    projections."""
    f, h = 64, 512
    gate = ggufgen.random_blocks(T_Q4_K, f * h, 5, 1)
    up = ggufgen.random_blocks(T_Q4_K, f * h, 5, 2)
    x = ggufgen.normal(h, 5, 3)
    L = _layout(T_Q4_K, 2 * f, h)
    rmap = np.array([(8 * (R // 16) + R % 16) if R % 16 < 8 else -1 - (8 * (R // 16) + R % 16 - 8)
                     for R in range(2 * f)], dtype=np.int32)
    packed = np.zeros(L.total_bytes, np.uint8)
    N.cuda().fl_repack(C.byref(L), gate.ctypes.data_as(C.c_void_p), up.ctypes.data_as(C.c_void_p),
                       rmap.ctypes.data_as(C.c_void_p), packed.ctypes.data_as(C.c_void_p), 2)
    y = np.zeros(2 * f, np.float32)
    N.cuda().fl_emulate_matvec(C.byref(L), packed.ctypes.data_as(C.c_void_p), x.ctypes.data_as(C.c_void_p),
                               y.ctypes.data_as(C.c_void_p))
    g_ref = O.matvec(T_Q4_K, gate, f, h, x)
    u_ref = O.matvec(T_Q4_K, up, f, h, x)
    y = y.reshape(-1, 16)
    np.testing.assert_allclose(y[:, :8].reshape(-1), g_ref, rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(y[:, 8:].reshape(-1), u_ref, rtol=1e-4, atol=2e-5)


def test_repack_thread_count_invariant():
    raw = ggufgen.random_blocks(T_Q6_K, 64 * 1024, 3, 3)
    L = _layout(T_Q6_K, 64, 1024)
    a = np.zeros(L.total_bytes, np.uint8)
    b = np.zeros(L.total_bytes, np.uint8)
    N.cuda().fl_repack(C.byref(L), raw.ctypes.data_as(C.c_void_p), None, None, a.ctypes.data_as(C.c_void_p), 1)
    N.cuda().fl_repack(C.byref(L), raw.ctypes.data_as(C.c_void_p), None, None, b.ctypes.data_as(C.c_void_p), 4)
    assert (a == b).all()


@pytest.mark.parametrize("t", TYPES + [0, 1, 30], ids=lambda t: str(t))
def test_generator_deterministic_and_decodable(t):
    n = 2048
    a = ggufgen.random_blocks(t, n, 42, 9)
    N.gen().gg_set_threads(1)
    b = ggufgen.random_blocks(t, n, 42, 9)
    N.gen().gg_set_threads(0)
    assert (a == b).all()
    rc, deq = O.dequantize(t, a)
    assert rc == O.OK
    x = ggufgen.normal(n, 42, 9, 0.02)
    # quantization error of the fitted blocks stays well inside the value range
    err = np.abs(deq - x)
    tol = {0: 0.0, 1: 1e-4, 30: 1e-3}.get(t, 0.02 * 0.35)
    assert err.max() <= tol + 1e-9, (TYPE_NAMES.get(t, t), err.max())


def test_normal_stream_moments():
    x = ggufgen.normal(1 << 20, 7, 1, 1.0).astype(np.float64)
    assert abs(x.mean()) < 5e-3 and abs(x.std() - 1.0) < 5e-3


def test_prompt_ids_in_range():
    p = ggufgen.prompt_ids(4096, 32000, 0)
    assert p.min() >= 0 and p.max() < 32000 and len(set(p.tolist())) > 3500
