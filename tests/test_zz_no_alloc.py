"""fl_topk_device, the allocation-free top-k (its scratch is a static device
array), against fl_topk, the session entry point, on the same logits.

It exists for callers that may not allocate device memory per call: an
engine whose device memory is one arena owned by its own pool, where a
cudaMalloc/cudaFree per token would synchronize the device and escape the
pool's accounting.

The file name sorts last, so in a full run it is collected after every other
test; it also passes alone.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import model_image
from dotnetfoundryllm_b200 import _native as N
from dotnetfoundryllm_b200 import ggufgen, loader, runtime


def test_sizes_outside_the_static_scratch_are_rejected():
    """Checked before any device work, so no GPU is needed."""
    lib = N.cuda()
    dummy = C.c_void_p(256)
    rc = lib.fl_topk_device(dummy, N.FL_TOPK_DEVICE_MAX_N + 1, 5, dummy, dummy, None)
    assert rc == N.FL_ERR_ARG
    assert "static top-k scratch" in N.last_error()
    assert lib.fl_topk_device(dummy, 100, 101, dummy, dummy, None) == N.FL_ERR_ARG
    assert lib.fl_topk_device(dummy, 100, 0, dummy, dummy, None) == N.FL_ERR_ARG
    assert lib.fl_topk_device(None, 100, 5, dummy, dummy, None) == N.FL_ERR_ARG


def _topk_device(d_logits, n: int, k: int):
    import torch
    d_ids = torch.full((k,), -1, dtype=torch.int32, device=d_logits.device)
    d_vals = torch.full((k,), float("nan"), dtype=torch.float32, device=d_logits.device)
    torch.cuda.synchronize()
    runtime.check(N.cuda().fl_topk_device(C.c_void_p(d_logits.data_ptr()), n, k, C.c_void_p(d_ids.data_ptr()),
                                          C.c_void_p(d_vals.data_ptr()), None), "fl_topk_device")
    torch.cuda.synchronize()
    return d_ids.cpu().numpy(), d_vals.cpu().numpy()


@pytest.mark.gpu
def test_matches_session_topk_on_two_calls_in_a_row():
    import torch
    model = loader.load(model_image("tiny"))
    fwd = runtime.CudaForwardPass(model)
    try:
        prompt = ggufgen.prompt_ids(4, model.desc.vocab, 7)
        kv = object()
        for i, tok in enumerate(prompt):
            fwd.forward(int(tok), i, kv)
        lg = fwd.logits.copy()
        d_logits = torch.from_numpy(lg).to("cuda:0")
        for k in (1, 5, 40, 1000):
            ref_ids, ref_vals, _ = fwd.topk(k)
            for _ in range(2):
                ids, vals = _topk_device(d_logits, lg.size, k)
                np.testing.assert_array_equal(ids, ref_ids)
                np.testing.assert_array_equal(vals, ref_vals)
    finally:
        fwd.close()
        model.close()


@pytest.mark.gpu
def test_largest_size_with_ties_matches_numpy():
    import torch
    n = N.FL_TOPK_DEVICE_MAX_N
    rng = np.random.default_rng(3)
    lg = rng.integers(-200, 200, n).astype(np.float32) / 8.0  # many ties
    d_logits = torch.from_numpy(lg).to("cuda:0")
    for k in (1, 64, 4096):
        order = np.lexsort((np.arange(n), -lg))[:k]
        for _ in range(2):
            ids, vals = _topk_device(d_logits, n, k)
            np.testing.assert_array_equal(ids, order)
            np.testing.assert_array_equal(vals, lg[order])


@pytest.mark.gpu
def test_flat_logits_at_the_largest_size_are_fast_and_in_index_order():
    """All n logits equal: every key ties with the k-th, so the selection is
    the first k indices.  The kernel takes the ties in index order with one
    block scan (no pairwise ranking), so this finishes in milliseconds even
    for k = n."""
    import time

    import torch
    n = N.FL_TOPK_DEVICE_MAX_N
    d_logits = torch.full((n,), 0.25, dtype=torch.float32, device="cuda:0")
    for k in (1, 40, 4096, n):
        _topk_device(d_logits, n, k)  # warm
        t0 = time.perf_counter()
        ids, vals = _topk_device(d_logits, n, k)
        dt = time.perf_counter() - t0
        np.testing.assert_array_equal(ids, np.arange(k))
        assert (vals == np.float32(0.25)).all()
        assert dt < 0.25, f"k={k}: {dt * 1e3:.1f} ms"


@pytest.mark.gpu
def test_signed_zeros_tie_and_go_by_index():
    """-0.0 and +0.0 compare equal (the reference's float compares), so among
    zeros the lower index comes first whatever the sign."""
    import torch
    lg = np.array([-0.0, 1.0, 0.0, -0.0, 0.0, -1.0, 0.0, -0.0], dtype=np.float32)
    d_logits = torch.from_numpy(lg).to("cuda:0")
    ids, vals = _topk_device(d_logits, lg.size, 6)
    np.testing.assert_array_equal(ids, [1, 0, 2, 3, 4, 6])
    np.testing.assert_array_equal(vals.view(np.uint32), lg[[1, 0, 2, 3, 4, 6]].view(np.uint32))
