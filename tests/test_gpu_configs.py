"""The BASELINE configurations at their real shapes, against the oracle.

Each model keeps its real hidden size, heads, head_dim, FFN width, vocabulary,
LM head, quantization types, RoPE base, sliding window and softcaps, with 2
decoder blocks instead of 32-42, so the CPU restatement finishes in seconds.
This covers what the tiny parity models cannot:
- 128k- and 256k-row LM heads (hundreds of row tiles per SM in the argmax);
- 4096-wide inputs and 14336-wide FFNs in the x encoding and the unit ranges;
- head_dim 128 and 256 at 8 kv heads;
- the 70B shapes: 8192-wide inputs and the 28672-wide input of the FFN down
  projection, more k-blocks than the token kernel's prologue keeps in
  registers (its one-k-block-at-a-time path).

Bars as everywhere: teacher-forced logits within 1e-3 + 1e-2*|ref|, through
the token loop and after the prompt path; greedy tokens identical.
"""
from __future__ import annotations

import dataclasses
import os

import numpy as np
import pytest

from dotnetfoundryllm_b200 import ggufgen, loader, runtime
from oracle import oracle as O

pytestmark = pytest.mark.gpu

PROMPT, N_GEN = 40, 6


@pytest.mark.parametrize("name", ["llama3-8b", "mistral-7b", "gemma2-9b", "llama3-70b"])
def test_real_shapes_match_the_oracle(name):
    spec = dataclasses.replace(ggufgen.SPECS[name], n_layers=2, ctx=512)
    img = ggufgen.build_model(spec)
    O.set_threads(os.cpu_count() or 1)
    m = O.Model(img)
    prompt = ggufgen.prompt_ids(PROMPT, m.vocab, 9)
    toks, logs = m.generate_greedy(prompt, N_GEN, collect_logits=True)
    m.close()
    model = loader.load(img, max_ctx=256)
    fwd = runtime.CudaForwardPass(model, max_ctx=256)
    try:
        feed = [int(prompt[-1])] + [int(t) for t in toks[:-1]]
        for path in ("token loop", "prompt path"):
            kv = object()
            if path == "token loop":
                for i in range(PROMPT - 1):
                    fwd.forward(int(prompt[i]), i, kv, want_logits=False)
            else:
                fwd.prefill(prompt[:-1], 0, kv)
            got = []
            for s, tok in enumerate(feed):
                am = fwd.forward(tok, PROMPT - 1 + s, kv)
                got.append(fwd.logits.copy())
                assert am == int(np.argmax(got[-1]))
            got = np.stack(got)
            err = np.abs(got - logs)
            bound = 1e-3 + 1e-2 * np.abs(logs)
            worst = np.unravel_index(np.argmax(err - bound), err.shape)
            assert (err <= bound).all(), f"{name} {path}: step {worst[0]} id {worst[1]}: {got[worst]} vs {logs[worst]}"
            for s in range(N_GEN):
                if int(np.argmax(got[s])) != int(toks[s]):
                    srt = np.sort(logs[s])
                    assert srt[-1] - srt[-2] < 1e-3, f"{name} {path}: greedy token {s} differs"
    finally:
        fwd.close()
        model.close()
