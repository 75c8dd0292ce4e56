"""The north-star model at full depth against the oracle.

Llama-3-8B architecture, all 32 decoder blocks, Q4_K matmuls with Q6_K for
attn_v, ffn_down and the LM head (vocab 128256): the model bench.py times.
The oracle keeps the quantized blocks and dequantizes each weight row where it
is used (the same floats as the reference's whole-tensor F32 load, so the same
results), which keeps host memory at the 4.9 GB of the file.

One 64-token random prompt, then 32 greedy tokens
(LlamaLanguageModel.GenerateAsync, LlamaLanguageModel.cs:126-216;
LlamaForwardPass.Forward, LlamaForwardPass.cs:82-130):
- the token loop (fl_forward per prompt token, then the 32 decode steps
  teacher-forced with the oracle's tokens): every step's logits within
  1e-3 + 1e-2*|ref| and its argmax equal to the oracle's token;
- the device-resident greedy loop (fl_decode_greedy) after the same prompt:
  all 32 generated ids identical to the oracle's;
- the prompt path (fl_prefill) followed by the same 32 teacher-forced steps,
  within the same bound.
"""
from __future__ import annotations

import dataclasses
import os

import numpy as np
import pytest

from dotnetfoundryllm_b200 import ggufgen, loader, runtime
from oracle import oracle as O

pytestmark = pytest.mark.gpu

PROMPT, N_GEN, CTX = 64, 32, 128


@pytest.fixture(scope="module")
def llama8b():
    spec = dataclasses.replace(ggufgen.SPECS["llama3-8b"], ctx=CTX)
    assert spec.n_layers == 32 and spec.hidden == 4096 and spec.vocab == 128256
    img = ggufgen.build_model(spec)
    O.set_threads(os.cpu_count() or 1)
    m = O.Model(img, lazy=True)
    prompt = ggufgen.prompt_ids(PROMPT, m.vocab, 0)
    toks, logs = m.generate_greedy(prompt, N_GEN, collect_logits=True)
    m.close()
    assert toks.size == N_GEN
    return img, prompt, toks, logs


def _check_steps(got: np.ndarray, logs: np.ndarray, toks: np.ndarray, what: str) -> None:
    err = np.abs(got - logs)
    bound = 1e-3 + 1e-2 * np.abs(logs)
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), f"{what}: step {worst[0]} id {worst[1]}: {got[worst]} vs {logs[worst]}"
    am = got.argmax(axis=1)
    assert (am == toks).all(), f"{what}: greedy ids differ at steps {np.nonzero(am != toks)[0].tolist()}"


def test_llama3_8b_full_depth_matches_the_oracle(llama8b):
    img, prompt, toks, logs = llama8b
    model = loader.load(img, max_ctx=CTX)
    fwd = runtime.CudaForwardPass(model, max_ctx=CTX)
    try:
        feed = [int(prompt[-1])] + [int(t) for t in toks[:-1]]

        # token loop, teacher-forced
        kv = object()
        for i in range(PROMPT - 1):
            fwd.forward(int(prompt[i]), i, kv, want_logits=False)
        got = []
        for s, tok in enumerate(feed):
            am = fwd.forward(tok, PROMPT - 1 + s, kv)
            got.append(fwd.logits.copy())
            assert am == int(np.argmax(got[-1]))
        _check_steps(np.stack(got), logs, toks, "token loop")

        # device greedy loop from the same prefix (positions 0..62 rewritten identically)
        for i in range(PROMPT - 1):
            fwd.forward(int(prompt[i]), i, kv, want_logits=False)
        ids = fwd.decode_greedy(int(prompt[-1]), PROMPT - 1, N_GEN)
        np.testing.assert_array_equal(ids, toks)

        # prompt path, then the teacher-forced steps
        kv2 = object()
        fwd.prefill(prompt[:-1], 0, kv2)
        got = []
        for s, tok in enumerate(feed):
            fwd.forward(tok, PROMPT - 1 + s, kv2)
            got.append(fwd.logits.copy())
        _check_steps(np.stack(got), logs, toks, "prompt path")
    finally:
        fwd.close()
        model.close()
