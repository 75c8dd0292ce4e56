"""Batched decode (fl_forward_batch) against the oracle: several sequences,
each in its own KV-cache slot, prompts through fl_prefill_seq, then batched
steps teacher-forced along each sequence's oracle greedy tokens.  Bars as for
the single-sequence path: logits within 1e-3 + 1e-2*|ref| (the split-fp16
GEMMs of the prompt path), greedy tokens identical."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import model_image
from dotnetfoundryllm_b200 import ggufgen, loader, runtime
from oracle import oracle as O

pytestmark = pytest.mark.gpu

N_GEN = 24
LENS = (9, 23, 14, 31)


def _ref(img, prompt):
    m = O.Model(img)
    try:
        return m.generate_greedy(prompt, N_GEN, collect_logits=True)
    finally:
        m.close()


@pytest.fixture(scope="module", params=["tiny", "tiny-mistral", "tiny-gemma2", "tiny-qwen2"])
def family(request):
    name = request.param
    img = model_image(name)
    model = loader.load(img)
    fwd = runtime.CudaForwardPass(model, max_ctx=256, max_batch=len(LENS))
    prompts = [ggufgen.prompt_ids(n, model.desc.vocab, 40 + i) for i, n in enumerate(LENS)]
    refs = [_ref(img, p) for p in prompts]
    yield name, model, fwd, prompts, refs
    fwd.close()
    model.close()


def _run(fwd, prompts, refs, order):
    """Teacher-forced batched decode; rows in `order`, slot = row's sequence."""
    B = len(order)
    for b in order:
        fwd.reset_slot(b)
        fwd.prefill_seq(b, prompts[b][:-1], 0)
    got_logits = np.zeros((len(prompts), N_GEN, fwd.vocab), np.float32)
    got_ids = np.zeros((len(prompts), N_GEN), np.int32)
    for step in range(N_GEN):
        toks = [int(prompts[b][-1]) if step == 0 else int(refs[b][0][step - 1]) for b in order]
        pos = [len(prompts[b]) - 1 + step for b in order]
        am, lg = fwd.forward_batch(toks, pos, list(order), want_logits=True)
        for r, b in enumerate(order):
            got_logits[b, step] = lg[r]
            got_ids[b, step] = am[r]
    return got_ids, got_logits


def test_batched_decode_matches_the_oracle(family):
    name, model, fwd, prompts, refs = family
    ids, lg = _run(fwd, prompts, refs, list(range(len(prompts))))
    for b, (toks, logs) in enumerate(refs):
        err = np.abs(lg[b] - logs)
        bound = 1e-3 + 1e-2 * np.abs(logs)
        worst = np.unravel_index(np.argmax(err - bound), err.shape)
        assert np.all(err <= bound), f"{name} seq {b}: step {worst[0]} id {worst[1]}: {lg[b][worst]} vs {logs[worst]}"
        for s in range(N_GEN):
            if ids[b, s] != toks[s]:
                srt = np.sort(logs[s])
                assert srt[-1] - srt[-2] < 1e-3, f"{name} seq {b} step {s}: {ids[b, s]} vs {toks[s]}"


def test_slots_are_independent_of_row_order(family):
    _, _, fwd, prompts, refs = family
    _, a = _run(fwd, prompts, refs, [0, 1, 2, 3])
    _, b = _run(fwd, prompts, refs, [2, 0, 3, 1])
    np.testing.assert_allclose(b, a, rtol=1e-4, atol=1e-4)
    _, c = _run(fwd, prompts, refs, [3, 1])
    np.testing.assert_allclose(c[[1, 3]], a[[1, 3]], rtol=1e-4, atol=1e-4)


def test_greedy_batch_completion(family):
    name, _, fwd, prompts, refs = family
    outs = runtime.generate_batch_greedy(fwd, prompts, N_GEN)
    for b, (toks, logs) in enumerate(refs):
        d = next((i for i in range(N_GEN) if outs[b][i] != toks[i]), None)
        if d is not None:
            srt = np.sort(logs[d])
            assert srt[-1] - srt[-2] < 1e-3, f"{name} seq {b}: token {d} differs"


def test_rewind_and_argument_errors(family):
    _, model, fwd, prompts, refs = family
    fwd.reset_slot(0)
    fwd.prefill_seq(0, prompts[0][:-1], 0)
    p = len(prompts[0]) - 1
    a = fwd.forward_batch([int(prompts[0][-1])], [p], [0], want_logits=True)[1]
    fwd.forward_batch([5], [p + 1], [0])
    b = fwd.forward_batch([int(prompts[0][-1])], [p], [0], want_logits=True)[1]  # rewinds slot 0
    np.testing.assert_allclose(b, a, rtol=1e-5, atol=1e-5)
    with pytest.raises(runtime.ArgumentError):
        fwd.forward_batch([1, 2], [0, 0], [1, 1])  # a slot twice
    with pytest.raises(runtime.ArgumentError):
        fwd.forward_batch([1], [p + 5], [0])  # skips cached positions
    with pytest.raises(runtime.ArgumentError):
        fwd.forward_batch([1], [0], [len(LENS)])  # no such slot
    with pytest.raises(runtime.ArgumentOutOfRangeError):
        fwd.forward_batch([model.desc.vocab], [0], [1])
