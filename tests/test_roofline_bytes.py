"""The decode roofline's numerator: the GGUF weight bytes one token streams.

Per decoded token the token loop reads every matrix and norm of the model once
plus one row of the token embedding (the embedding phase dequantizes only the
row of the current token).  These figures are the algorithmic bytes the bench
divides by the token kernel's launch time, before the K/V rows are added; they
follow from the configurations' shapes and quantization types alone, so the
generator's tensor plan is checked against them here on the CPU.
"""
from __future__ import annotations

import pytest

from dotnetfoundryllm_b200 import gguf, ggufgen

# bytes per decoded token: all tensors but token_embd, plus one token_embd row
EXPECTED = {
    "tiny": 26_156_452,           # layers 12,681,216 + head 13,440,000 + norms 34,816 + embedding row 420
    "llama3-8b": 4_876_921_088,   # layers + norms 4,445,962,240; head 430,940,160; output_norm 16,384; row 2,304
    "mistral-7b": 7_555_862_784,  # Q8_0 matrices 7,554,793,472 + norms 1,064,960 + embedding row 4,352
    "gemma2-9b": 6_477_538_172,
    "llama3-70b": 39_099_994_624,
}


def token_bytes(spec: ggufgen.ModelSpec) -> int:
    total = 0
    for name, dims, t, _ in ggufgen.tensor_plan(spec):
        elems_per_block, block_bytes = gguf.BLOCK[t]
        if name == "token_embd.weight":
            total += dims[0] // elems_per_block * block_bytes  # one row of `hidden` values
            continue
        n = 1
        for d in dims:
            n *= d
        assert n % elems_per_block == 0, name
        total += n // elems_per_block * block_bytes
    return total


@pytest.mark.parametrize("name", sorted(EXPECTED))
def test_weight_bytes_per_token(name):
    assert token_bytes(ggufgen.SPECS[name]) == EXPECTED[name]
