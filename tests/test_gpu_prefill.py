"""The prompt path (fl_prefill) against the CPU restatement.

The reference feeds prompt tokens one at a time (LlamaLanguageModel.cs:
133-137).  fl_prefill runs all prompt tokens of a chunk through each layer
together, with fp16 tensor-core GEMMs for the projections.  The K/V it leaves
in the cache must let decoding continue exactly as after the token-by-token
prefill: under teacher forcing every decode step's logits are within
1e-3 + 1e-2·|ref| of the oracle's, and greedy tokens are identical.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import model_image
from dotnetfoundryllm_b200 import ggufgen, loader, runtime
from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 1e-3
N_PROMPT, N_GEN = 64, 64
_REF: dict = {}


def reference(name: str):
    if name not in _REF:
        m = O.Model(model_image(name))
        prompt = ggufgen.prompt_ids(N_PROMPT, m.vocab, 2)
        toks, logs = m.generate_greedy(prompt, N_GEN, collect_logits=True)
        _REF[name] = (prompt, toks, logs)
        m.close()
    return _REF[name]


@pytest.fixture(scope="module", params=["tiny", "tiny-mistral", "tiny-gemma2", "tiny-qwen2"])
def family(request):
    model = loader.load(model_image(request.param))
    fwd = runtime.CudaForwardPass(model)
    yield request.param, model, fwd
    fwd.close()
    model.close()


def _decode_after_prefill(fwd, prompt, feed, splits=()):
    kv = object()
    bounds = [0, *splits, len(prompt) - 1]
    for a, b in zip(bounds[:-1], bounds[1:]):
        fwd.prefill(prompt[a:b], a, kv)
    pos = len(prompt) - 1
    logits, am = [], []
    for tok in feed:
        am.append(fwd.forward(int(tok), pos, kv))
        logits.append(fwd.logits.copy())
        pos += 1
    return np.stack(logits), np.array(am)


def test_decode_after_prefill_matches_the_oracle(family):
    name, model, fwd = family
    prompt, toks, logs = reference(name)
    feed = [int(prompt[-1])] + [int(t) for t in toks[:-1]]
    got, am = _decode_after_prefill(fwd, prompt, feed)
    err = np.abs(got - logs)
    bound = ATOL + RTOL * np.abs(logs)
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), f"{name}: step {worst[0]} id {worst[1]}: {got[worst]} vs {logs[worst]}"
    assert (am == np.argmax(got, axis=1)).all()


def test_greedy_tokens_after_prefill(family):
    name, model, fwd = family
    prompt, toks, logs = reference(name)
    kv = object()
    fwd.prefill(prompt[:-1], 0, kv)
    got = fwd.decode_greedy(int(prompt[-1]), len(prompt) - 1, N_GEN)
    diverge = next((i for i in range(len(toks)) if got[i] != toks[i]), None)
    if diverge is not None:
        s = np.sort(logs[diverge])
        assert diverge >= 32, f"{name}: token {diverge} differs (reference top-2 gap {s[-1] - s[-2]:.3e})"


def test_chunked_prefill_equals_one_pass(family):
    """Two calls (the second attends to the first's cached keys) = one call,
    up to summation order: attention's score rows span a different number of
    cached keys, so logits may differ by a few 1e-5."""
    name, model, fwd = family
    prompt, toks, logs = reference(name)
    feed = [int(prompt[-1])] + [int(t) for t in toks[:7]]
    one, _ = _decode_after_prefill(fwd, prompt, feed)
    two, _ = _decode_after_prefill(fwd, prompt, feed, splits=(23,))
    np.testing.assert_allclose(two, one, rtol=1e-4, atol=1e-4)


def test_prefill_argument_errors(family):
    name, model, fwd = family
    with pytest.raises(runtime.ArgumentOutOfRangeError):
        fwd.prefill([1, model.desc.vocab], 0, object())
    kv = object()
    fwd.prefill([1, 2, 3], 0, kv)
    with pytest.raises(runtime.ArgumentError):
        fwd.prefill([4], 5, kv)  # skips cached positions


@pytest.mark.parametrize("t", [12, 13, 14, 8, 2])  # Q4_K, Q5_K, Q6_K, Q8_0, Q4_0
def test_split_weights_are_the_exact_values(t):
    """The prefill's weight layout: every value bit-exactly dequantized, times
    FL_PF_WSCALE, as fp16 hi and lo = fp16(v - hi), in [hi | lo | hi]."""
    import ctypes as C
    from dotnetfoundryllm_b200 import _native as N
    from oracle import oracle as O
    rows, cols = 48, 768
    raw = ggufgen.random_blocks(t, rows * cols, 5, t)
    # random bytes as well: every bit pattern of the scales and quants
    raw2 = np.random.default_rng(t).integers(0, 256, raw.size, dtype=np.uint8)
    for blob in (raw, raw2):
        out = np.zeros(rows * cols * 3, dtype=np.uint16)
        runtime.check(N.cuda().fl_dequant_split_test(t, blob.ctypes.data_as(C.c_void_p), blob.size, rows, cols,
                                                     out.ctypes.data_as(C.c_void_p)), "fl_dequant_split_test")
        rc, v = O.dequantize(t, blob, rows * cols)
        assert rc == O.OK
        x = (v.astype(np.float32) * np.float32(256.0)).reshape(rows, cols)
        with np.errstate(over="ignore", invalid="ignore"):  # random bytes: values past the fp16 range
            hi = x.astype(np.float16)
            lo = (x - hi.astype(np.float32)).astype(np.float16)
        got = out.view(np.float16).reshape(rows, 3 * cols)
        finite = np.isfinite(x)
        for part, want in ((0, hi), (1, lo), (2, hi)):
            g = got[:, part * cols:(part + 1) * cols]
            np.testing.assert_array_equal(g.view(np.uint16)[finite], want.view(np.uint16)[finite])


def test_weight_past_the_fp16_range_is_reported_not_stored_as_infinity():
    """The prompt path's tensor-core operands are fp16 (weights times
    FL_PF_WSCALE = 256): a weight of magnitude > 255.9 cannot be represented.
    fl_prefill reports it (FL_ERR_UNSUPPORTED, NotSupportedError) instead of
    computing with infinities, the cache keeps only the positions before the
    prompt, and the token loop (no such limit) runs the same tokens."""
    from dotnetfoundryllm_b200 import gguf
    img = model_image("tiny").copy()
    g = gguf.parse(img)
    t = g.find_tensor("blk.0.attn_q.weight")
    assert t.type == 12  # Q4_K: f16 d at byte 0 of each 144-byte block
    off = g.data_start + t.offset
    img[off:off + 2] = np.frombuffer(np.float16(60000.0).tobytes(), np.uint8)  # d * scale * q >> 256
    model = loader.load(img, max_ctx=64)
    fwd = runtime.CudaForwardPass(model, max_ctx=64)
    try:
        kv = object()
        with pytest.raises(runtime.NotSupportedError, match="fp16 range"):
            fwd.prefill([1, 2, 3, 4], 0, kv)
        with pytest.raises(runtime.ArgumentError):
            fwd.forward(5, 4, kv)  # nothing of the refused prompt is cached
        for i, tok in enumerate([1, 2, 3, 4]):
            fwd.forward(tok, i, kv, want_logits=False)
    finally:
        fwd.close()
        model.close()
