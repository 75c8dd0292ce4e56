"""The oracle's row-wise weight decoding (``Model(lazy=True)``, used for the
full-depth 8B parity test) gives bit-identical logits and tokens to the
reference's whole-tensor F32 load (GgufModelLoader.LoadTensor,
GgufModelLoader.cs:409-418), on every tiny family."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import model_image
from dotnetfoundryllm_b200 import ggufgen
from oracle import oracle as O


@pytest.mark.parametrize("name", ["tiny", "tiny-mistral", "tiny-gemma2", "tiny-qwen2"])
def test_lazy_rows_are_bit_identical(name):
    img = model_image(name)
    eager, lazy = O.Model(img), O.Model(img, lazy=True)
    try:
        prompt = ggufgen.prompt_ids(12, eager.vocab, 5)
        ta, la = eager.generate_greedy(prompt, 6, collect_logits=True)
        tb, lb = lazy.generate_greedy(prompt, 6, collect_logits=True)
        np.testing.assert_array_equal(ta, tb)
        np.testing.assert_array_equal(la.view(np.uint32), lb.view(np.uint32))
    finally:
        eager.close()
        lazy.close()
