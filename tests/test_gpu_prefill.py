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
    up to summation order: the GEMM library picks its reduction split per
    shape, so logits may differ by a few 1e-5."""
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
