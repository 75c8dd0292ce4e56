"""Writes tests/golden/reference_kats.json: the known-answer vectors held by the
reference's own xUnit tests for the token-loop path, each with the file:line it
comes from (paths inside justinamiller/DotNetFoundryLLM v1.0.0).

The reference is C#/.NET 10 and cannot run here, so the vectors are transcribed
from the test sources.  When the reference source tree is given (the
REFERENCE_ROOT environment variable, or --reference DIR), every entry's
`needle` strings are checked against the cited lines so a transcription error
fails loudly.

    python tests/golden/make_reference_kats.py [--reference DIR] [--check-only]
"""
from __future__ import annotations

import json
import struct
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def _reference_root() -> Path | None:
    if "--reference" in sys.argv:
        return Path(sys.argv[sys.argv.index("--reference") + 1])
    env = os.environ.get("REFERENCE_ROOT")
    return Path(env) if env else None


REF = _reference_root()
DQ = "tests/DotNetFoundryLLM.Quantization.Tests/DequantizerTests.cs"
GS = "tests/DotNetFoundryLLM.Sampling.Tests/GreedySamplerTests.cs"
TK = "tests/DotNetFoundryLLM.Sampling.Tests/TopKSamplerTests.cs"
GR = "tests/DotNetFoundryLLM.ModelFormats.Gguf.Tests/GgufReaderTests.cs"
TO = "tests/DotNetFoundryLLM.Tensors.Tests/TensorOperationsTests.cs"

KATS = {
    "half_to_float": [
        {"bits": 0x0000, "value": 0.0, "src": f"{DQ}:15", "needle": ["0x0000"]},
        {"bits": 0x3C00, "value": 1.0, "src": f"{DQ}:22", "needle": ["0x3C00"]},
        {"bits": 0xBC00, "value": -1.0, "src": f"{DQ}:29", "needle": ["0xBC00"]},
    ],
    "bf16_to_float": [
        {"bits": 0x0000, "value": 0.0, "src": f"{DQ}:37", "needle": ["0x0000"]},
        {"bits": 0x3F80, "value": 1.0, "src": f"{DQ}:44", "needle": ["0x3F80"]},
        {"bits": 0x4000, "value": 2.0, "src": f"{DQ}:51", "needle": ["0x4000"]},
    ],
    # blocks given as hex strings; expected values as {index: value} (others unchecked unless "all")
    "dequantize": [
        {"name": "F32 round trip", "type": 0, "hex": struct.pack("<4f", 1.5, -2.25, 0.0, 3.14).hex(),
         "expect_all": [1.5, -2.25, 0.0, 3.14], "src": f"{DQ}:59", "needle": ["1.5f, -2.25f, 0f, 3.14f"]},
        {"name": "F16 known", "type": 1, "hex": "003c00bc", "expect_all": [1.0, -1.0], "src": f"{DQ}:87",
         "needle": ["0x3C00"]},
        {"name": "BF16 known", "type": 30, "hex": "803f0040", "expect_all": [1.0, 2.0], "src": f"{DQ}:103",
         "needle": ["0x3F80"]},
        {"name": "Q4_0 zero block", "type": 2, "hex": "0000" + "88" * 16, "expect_all": [0.0] * 32,
         "src": f"{DQ}:124", "needle": ["0x88"]},
        {"name": "Q4_0 known block", "type": 2, "hex": "003c79" + "88" * 15, "expect": {"0": 1.0, "16": -1.0, "1": 0.0},
         "src": f"{DQ}:144", "needle": ["0x79"]},
        {"name": "Q8_0 known block", "type": 8, "hex": "003c" + "ff0001" + "00" * 29,
         "expect": {"0": -1.0, "1": 0.0, "2": 1.0}, "src": f"{DQ}:174", "needle": ["-1"]},
        {"name": "Q4_K zero block", "type": 12, "hex": "003c0000" + "00" * 140, "expect_all": [0.0] * 256,
         "src": f"{DQ}:242", "needle": ["0x3C00"]},
        {"name": "Q5_K zero block", "type": 13, "hex": "003c0000" + "00" * 172, "expect_all": [0.0] * 256,
         "src": f"{DQ}:259", "needle": ["0x3C00"]},
    ],
    "dequantize_throws": [
        {"type": 0, "src_len": 5, "dst_len": 1, "exception": "ArgumentException", "src": f"{DQ}:77",
         "needle": ["new byte[5]"]},
        {"type": 2, "src_len": 17, "dst_len": 32, "exception": "ArgumentException", "src": f"{DQ}:163",
         "needle": ["new byte[17]"]},
        {"type": 8, "src_len": 33, "dst_len": 32, "exception": "ArgumentException", "src": f"{DQ}:190",
         "needle": ["new byte[33]"]},
        {"type": 99, "src_len": 4, "dst_len": 1, "exception": "NotSupportedException", "src": f"{DQ}:196",
         "needle": ["99"]},
        {"type": 12, "src_len": 143, "dst_len": 256, "exception": "ArgumentException", "src": f"{DQ}:275",
         "needle": ["new byte[143]"]},
        {"type": 13, "src_len": 175, "dst_len": 256, "exception": "ArgumentException", "src": f"{DQ}:282",
         "needle": ["new byte[175]"]},
    ],
    "element_count": [
        {"type": 0, "bytes": 16, "count": 4, "src": f"{DQ}:206", "needle": ["ElementCount(0, 16)"]},
        {"type": 2, "bytes": 18, "count": 32, "src": f"{DQ}:213", "needle": ["ElementCount(2, 18)"]},
        {"type": 8, "bytes": 34, "count": 32, "src": f"{DQ}:220", "needle": ["ElementCount(8, 34)"]},
        {"type": 12, "bytes": 144, "count": 256, "src": f"{DQ}:227", "needle": ["ElementCount(12, 144)"]},
        {"type": 13, "bytes": 176, "count": 256, "src": f"{DQ}:234", "needle": ["ElementCount(13, 176)"]},
    ],
    "argmax": [
        {"x": [0.1, 5.0, 0.3, 0.2], "index": 1, "src": f"{GS}:14", "needle": ["0.1f, 5.0f, 0.3f, 0.2f"]},
        {"x": [100.0, 0.0, -1.0], "index": 0, "src": f"{GS}:22", "needle": ["100f, 0f, -1f"]},
        {"x": [-1.0, 0.0, 99.0], "index": 2, "src": f"{GS}:29", "needle": ["-1f, 0f, 99f"]},
        {"x": [42.0], "index": 0, "src": f"{GS}:36", "needle": ["42f"]},
    ],
    "apply_topk": [
        {"x": [1.0, 5.0, 0.5, 3.0], "k": 2, "neg_inf": [0, 2], "kept": [1, 3], "src": f"{TK}:47",
         "needle": ["1f, 5f, 0.5f, 3f"]},
        {"x": [1.0, 2.0, 3.0], "k": 10, "neg_inf": [], "kept": [0, 1, 2], "src": f"{TK}:59",
         "needle": ["1f, 2f, 3f"]},
    ],
    "dot": [
        {"a": [1.0, 2.0, 3.0], "b": [4.0, 5.0, 6.0], "value": 32.0, "src": f"{TO}:71", "needle": ["1f, 2f, 3f"]},
    ],
    "gguf_reader": [
        {"case": "invalid_magic", "src": f"{GR}:42", "needle": ["0x00, 0x01, 0x02, 0x03"]},
        {"case": "invalid_versions", "versions": [0, 1, 4], "src": f"{GR}:48", "needle": ["InlineData(0u)"]},
        {"case": "empty", "versions": [2, 3], "src": f"{GR}:61", "needle": ["InlineData(2u)"]},
        {"case": "string_meta", "key": "general.architecture", "value": "llama", "src": f"{GR}:87",
         "needle": ["general.architecture"]},
        {"case": "uint32_meta", "key": "llama.block_count", "value": 32, "src": f"{GR}:109",
         "needle": ["llama.block_count"]},
        {"case": "string_array", "key": "tokenizer.ggml.tokens", "value": ["hello", "world"], "src": f"{GR}:130",
         "needle": ["tokenizer.ggml.tokens"]},
        {"case": "tensor_info", "name": "output_norm.weight", "dims": [4096], "type": 0, "offset": 0,
         "src": f"{GR}:156", "needle": ["output_norm.weight"]},
        {"case": "find_tensor", "name": "token_embd.weight", "dims": [32000, 4096], "type": 0, "src": f"{GR}:183",
         "needle": ["token_embd.weight"]},
    ],
}


def check_against_reference() -> list[str]:
    problems = []
    if REF is None or not REF.exists():
        print("reference tree not given: the citations are not re-checked")
        return problems
    for group in KATS.values():
        for e in group:
            path, line = e["src"].rsplit(":", 1)
            p = REF / path
            if not p.exists():
                problems.append(f"{e['src']}: file missing")
                continue
            lines = p.read_text().splitlines()
            lo, hi = max(0, int(line) - 3), min(len(lines), int(line) + 3)
            window = "\n".join(lines[lo:hi])
            for n in e.get("needle", []):
                if n not in window:
                    problems.append(f"{e['src']}: '{n}' not found near the cited line")
    return problems


def main() -> int:
    problems = check_against_reference()
    for p in problems:
        print("MISMATCH", p)
    if problems:
        return 1
    if "--check-only" not in sys.argv:
        out = {k: [{kk: vv for kk, vv in e.items() if kk != "needle"} for e in v] for k, v in KATS.items()}
        (HERE / "reference_kats.json").write_text(json.dumps(out, indent=1) + "\n")
        print("wrote", HERE / "reference_kats.json")
    return 0


if __name__ == "__main__":
    sys.exit(main())
