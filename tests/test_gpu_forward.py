"""End-to-end parity of the device token loop against the CPU restatement.

For each model family (tiny Llama-3 = BASELINE config 0, small Mistral /
Gemma 2 variants whose sliding windows bind, and a small Qwen2 with QKV biases
and a 7-way query-head group), a seeded GGUF is loaded twice:
by the oracle (F32 weights, LlamaForwardPass & co.) and through
fl_model_upload (raw blocks).  The greedy generation loop of
LlamaLanguageModel.GenerateAsync runs on both; the criteria are those of the
north star:

- logits at every decode step within 1e-2 relative / 1e-3 absolute
  (|gpu - ref| <= 1e-3 + 1e-2 * |ref|), checked under teacher forcing so every
  one of the 128 steps is compared even if a near-tie flips a token;
- greedy token ids identical for at least the first 32 generated tokens (all
  128 are expected; a divergence reports the reference's top-2 gap).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import model_image
from dotnetfoundryllm_b200 import ggufgen, loader, runtime
from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 1e-3
N_PROMPT, N_GEN = 64, 128

_REF: dict = {}


def reference(name: str):
    """Oracle greedy run: (prompt, tokens, logits[steps, vocab])."""
    if name not in _REF:
        img = model_image(name)
        m = O.Model(img)
        prompt = ggufgen.prompt_ids(N_PROMPT, m.vocab, 0)
        toks, logs = m.generate_greedy(prompt, N_GEN, collect_logits=True)
        _REF[name] = (prompt, toks, logs, m.eos)
        m.close()
    return _REF[name]


def _teacher_forced_logits(fwd: runtime.CudaForwardPass, prompt, ref_tokens):
    kv = object()
    pos = 0
    for i in range(len(prompt) - 1):
        fwd.forward(int(prompt[i]), pos, kv, want_logits=False)
        pos += 1
    feed = [int(prompt[-1])] + [int(t) for t in ref_tokens[:-1]]
    out, am = [], []
    for tok in feed:
        am.append(fwd.forward(tok, pos, kv))
        out.append(fwd.logits.copy())
        pos += 1
    return np.stack(out), np.array(am)


@pytest.fixture(scope="module", params=["tiny", "tiny-mistral", "tiny-gemma2", "tiny-qwen2"])
def family(request):
    name = request.param
    prompt, toks, logs, eos = reference(name)
    model = loader.load(model_image(name))
    fwd = runtime.CudaForwardPass(model)
    yield name, model, fwd, prompt, toks, logs, eos
    fwd.close()
    model.close()


def test_logits_within_tolerance_every_step(family):
    name, model, fwd, prompt, toks, logs, eos = family
    got, am = _teacher_forced_logits(fwd, prompt, toks)
    assert got.shape == logs.shape
    err = np.abs(got - logs)
    bound = ATOL + RTOL * np.abs(logs)
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), f"{name}: step {worst[0]} id {worst[1]}: {got[worst]} vs {logs[worst]}"
    # the device argmax is TensorPrimitives.IndexOfMax of the device logits
    assert (am == np.argmax(got, axis=1)).all()


def test_greedy_tokens_identical(family):
    name, model, fwd, prompt, toks, logs, eos = family
    got, _ = runtime.generate_greedy(fwd, prompt, N_GEN, eos=eos)
    n = min(len(got), len(toks))
    diverge = next((i for i in range(n) if got[i] != toks[i]), None)
    if diverge is not None:
        s = np.sort(logs[diverge])
        gap = s[-1] - s[-2]
        assert diverge >= 32, f"{name}: token {diverge} differs (reference top-2 gap {gap:.3e})"
        pytest.xfail(f"{name}: tokens identical for {diverge} steps; step {diverge} is a near tie ({gap:.3e})")
    assert len(got) == len(toks)


def test_device_greedy_loop_matches_host_loop(family):
    name, model, fwd, prompt, toks, logs, eos = family
    kv = object()
    pos = 0
    for i in range(len(prompt) - 1):
        fwd.forward(int(prompt[i]), pos, kv, want_logits=False)
        pos += 1
    dev = fwd.decode_greedy(int(prompt[-1]), pos, 32)
    host, _ = runtime.generate_greedy(fwd, prompt, 32)
    np.testing.assert_array_equal(dev, host[:32])


def test_topk_matches_numpy(family):
    name, model, fwd, prompt, toks, logs, eos = family
    fwd.forward(int(prompt[0]), 0, object())
    lg = fwd.logits.copy()
    for k in (1, 5, 40):
        ids, vals, thr = fwd.topk(k)
        order = np.lexsort((np.arange(lg.size), -lg))[:k]
        np.testing.assert_array_equal(ids, order)
        np.testing.assert_array_equal(vals, lg[order])
        assert thr == lg[order[-1]]


def test_argument_errors(family):
    name, model, fwd, prompt, toks, logs, eos = family
    with pytest.raises(runtime.ArgumentOutOfRangeError):
        fwd.forward(model.desc.vocab, 0, object())
    with pytest.raises(runtime.ArgumentOutOfRangeError):
        fwd.forward(-1, 0, object())
    kv = object()
    fwd.forward(1, 0, kv)
    with pytest.raises(runtime.ArgumentError):
        fwd.forward(1, 5, kv)  # skips cached positions
    with pytest.raises(runtime.ArgumentError):
        fwd.forward(1, model.desc.max_ctx, kv)


def test_profile_step_phases(family):
    """One persistent launch per token; the per-phase stamps cover the step."""
    name, model, fwd, prompt, toks, logs, eos = family
    fwd.forward(1, 0, object())
    p = fwd.profile_step(2, 1)
    assert p["launches"] == 1
    assert fwd.launches_per_step() == 1
    assert p["ms"]["step"] > 0
    assert p["ms"]["matvec"] > 0 and p["ms"]["attention"] > 0
    assert abs(p["ms"]["step"] - sum(p["ms"][k] for k in ("matvec", "attention", "other"))) < 1e-6
    assert p["bytes"]["matvec"] > 0.9 * model.weight_bytes() - 1e6


def test_missing_tensor_is_reported():
    img = model_image("tiny")
    from dotnetfoundryllm_b200 import gguf
    g = gguf.parse(img)
    model = runtime.CudaModel(loader.build_desc(g))
    try:
        for t in g.tensors:
            if t.name != "blk.3.ffn_down.weight":
                model.upload(t.name, t.type, t.dims, g.tensor_bytes(t))
        with pytest.raises(runtime.InvalidOperationError, match="blk.3.ffn_down.weight"):
            model.finalize()
    finally:
        model.close()


def test_tied_output_falls_back_to_embedding():
    """GgufModelLoader: output.weight absent → the token embedding is the LM head."""
    img = model_image("tiny")
    from dotnetfoundryllm_b200 import gguf
    g = gguf.parse(img)
    w = ggufgen.build_writer(ggufgen.SPECS["tiny"])
    w.tensors = [t for t in w.tensors if t.name != "output.weight"]
    img2 = w.build()
    m = O.Model(img2)
    prompt = ggufgen.prompt_ids(8, m.vocab, 3)
    toks, logs = m.generate_greedy(prompt, 8, collect_logits=True)
    m.close()
    model = loader.load(img2)
    fwd = runtime.CudaForwardPass(model)
    got, glogs = runtime.generate_greedy(fwd, prompt, 8, collect_logits=True)
    fwd.close()
    model.close()
    np.testing.assert_array_equal(got, toks)
    assert (np.abs(glogs - logs) <= ATOL + RTOL * np.abs(logs)).all()
