"""Seeded random-init GGUF models for the benchmark configurations.

The reference ships no model files, so the tests and the benchmark build
their models here: weights from a counter-based N(0, sigma) stream
(``csrc/ggufgen.c``), quantized with the inverse of the reference decoder,
norm weights 1.0, metadata written exactly as ``GgufModelLoader`` reads it
(src/DotNetFoundryLLM.ModelFormats.Gguf/GgufModelLoader.cs:104-334):

- ``{arch}.*`` hyper-parameters as UInt32, RoPE base and softcaps as Float32
  (``GetFloat`` accepts Float32 only, :472-478);
- ``tokenizer.ggml.tokens`` (the loader refuses a model without a vocabulary,
  :378-381) with placeholder strings;
- Gemma 2: ``gemma2.attention.key_length`` is written (256 != 3584/16) and
  ``query_pre_attn_scalar`` is omitted, so the scale is 1/sqrt(head_dim).
"""
from __future__ import annotations

import ctypes as C
import zlib
from dataclasses import dataclass, field

import numpy as np

from . import _native
from .gguf import (ARR, F32, STR, T_F32, T_Q4_K, T_Q5_K, T_Q6_K, T_Q8_0, U32, GgufWriter)


@dataclass
class ModelSpec:
    name: str
    arch: str                 # llama | mistral | gemma2 | qwen2
    n_layers: int
    hidden: int
    n_heads: int
    n_kv: int
    ffn: int
    vocab: int
    ctx: int
    rope_base: float = 10000.0
    head_dim: int | None = None          # gemma2 key_length
    window: int | None = None            # mistral / gemma2 sliding window
    attn_softcap: float | None = None
    final_softcap: float | None = None
    types: dict = field(default_factory=dict)   # role -> ggml type
    sigma: float = 0.02
    seed: int = 0
    bos: int = 1
    eos: int = 2

    def type_of(self, role: str) -> int:
        return self.types.get(role, self.types.get("matmul", T_Q4_K))

    @property
    def hd(self) -> int:
        return self.head_dim or self.hidden // self.n_heads


def _llama_types(**kw):
    return dict(kw)


SPECS = {
    # tiny Llama-3 (CPU-runnable reference)
    "tiny": ModelSpec("tiny-llama3", "llama", 8, 512, 8, 2, 1408, 32000, 512, rope_base=500000.0,
                      types=_llama_types(matmul=T_Q4_K, token_embd=T_Q6_K, output=T_Q6_K)),
    # Llama-3-8B Q4_K_M-style
    "llama3-8b": ModelSpec("llama3-8b", "llama", 32, 4096, 32, 8, 14336, 128256, 8192, rope_base=500000.0,
                           types=_llama_types(matmul=T_Q4_K, token_embd=T_Q4_K, attn_v=T_Q6_K, ffn_down=T_Q6_K,
                                              output=T_Q6_K)),
    # Mistral-7B Q8_0, window 4096
    "mistral-7b": ModelSpec("mistral-7b", "mistral", 32, 4096, 32, 8, 14336, 32000, 4096, rope_base=1000000.0,
                            window=4096, types=_llama_types(matmul=T_Q8_0, token_embd=T_Q8_0, output=T_Q8_0)),
    # Gemma-2-9B, Q5_K matmuls, Q6_K embedding/output
    "gemma2-9b": ModelSpec("gemma2-9b", "gemma2", 42, 3584, 16, 8, 14336, 256000, 8192, head_dim=256,
                           window=4096, attn_softcap=50.0, final_softcap=30.0,
                           types=_llama_types(matmul=T_Q5_K, token_embd=T_Q6_K, output=T_Q6_K)),
    # Llama-3-70B, all Q4_K
    "llama3-70b": ModelSpec("llama3-70b", "llama", 80, 8192, 64, 8, 28672, 128256, 16384, rope_base=500000.0,
                            types=_llama_types(matmul=T_Q4_K, token_embd=T_Q4_K, output=T_Q4_K)),
    # small variants of the other families for the parity tests
    "tiny-mistral": ModelSpec("tiny-mistral", "mistral", 4, 512, 8, 2, 1408, 32000, 512, rope_base=1000000.0,
                              window=48, types=_llama_types(matmul=T_Q8_0, token_embd=T_Q8_0, output=T_Q8_0)),
    # Qwen2 (QKV biases) with Qwen2-7B's 7-way query-head group (28/4 there,
    # 14/2 here); hidden 896 and FFN 2432 are not multiples of 256, so the
    # K-quant rows straddle blocks (expanded headers)
    "tiny-qwen2": ModelSpec("tiny-qwen2", "qwen2", 4, 896, 14, 2, 2432, 32000, 512, rope_base=1000000.0,
                            types=_llama_types(matmul=T_Q4_K, attn_v=T_Q6_K, ffn_down=T_Q6_K, token_embd=T_Q6_K,
                                               output=T_Q6_K)),
    # tensor-parallel parity: every split (heads, FFN rows, vocabulary, Wo/down
    # columns in whole 256-blocks) divides for 2, 4 and 8 ranks
    "small-tp": ModelSpec("small-tp", "llama", 2, 2048, 16, 8, 4096, 32000, 512, rope_base=500000.0,
                          types=_llama_types(matmul=T_Q4_K, token_embd=T_Q6_K, attn_v=T_Q6_K, ffn_down=T_Q6_K,
                                             output=T_Q6_K)),
    "tiny-gemma2": ModelSpec("tiny-gemma2", "gemma2", 4, 512, 4, 2, 1536, 32000, 512, head_dim=256, window=40,
                             attn_softcap=50.0, final_softcap=30.0,
                             types=_llama_types(matmul=T_Q5_K, token_embd=T_Q6_K, output=T_Q6_K)),
}


def stream_id(name: str) -> int:
    return zlib.crc32(name.encode()) | (len(name) << 32)


def tensor_plan(spec: ModelSpec) -> list[tuple[str, list[int], int, str]]:
    """(name, GGUF dims [ne0=cols, ne1=rows], type, kind) per tensor, in the
    loader's order (GgufModelLoader.LoadWeights :336-372)."""
    h, f, V = spec.hidden, spec.ffn, spec.vocab
    qd, kvd = spec.n_heads * spec.hd, spec.n_kv * spec.hd
    out = [("token_embd.weight", [h, V], spec.type_of("token_embd"), "w")]
    for i in range(spec.n_layers):
        p = f"blk.{i}."
        out.append((p + "attn_norm.weight", [h], T_F32, "one"))
        if spec.arch == "gemma2":
            out.append((p + "post_attn_norm.weight", [h], T_F32, "one"))
        out.append((p + "attn_q.weight", [h, qd], spec.type_of("attn_q"), "w"))
        out.append((p + "attn_k.weight", [h, kvd], spec.type_of("attn_k"), "w"))
        out.append((p + "attn_v.weight", [h, kvd], spec.type_of("attn_v"), "w"))
        out.append((p + "attn_output.weight", [qd, h], spec.type_of("attn_output"), "w"))
        if spec.arch == "qwen2":
            out.append((p + "attn_q.bias", [qd], T_F32, "w"))
            out.append((p + "attn_k.bias", [kvd], T_F32, "w"))
            out.append((p + "attn_v.bias", [kvd], T_F32, "w"))
        out.append((p + "ffn_norm.weight", [h], T_F32, "one"))
        if spec.arch == "gemma2":
            out.append((p + "post_ffn_norm.weight", [h], T_F32, "one"))
        out.append((p + "ffn_gate.weight", [h, f], spec.type_of("ffn_gate"), "w"))
        out.append((p + "ffn_up.weight", [h, f], spec.type_of("ffn_up"), "w"))
        out.append((p + "ffn_down.weight", [f, h], spec.type_of("ffn_down"), "w"))
    out.append(("output_norm.weight", [h], T_F32, "one"))
    if spec.type_of("output") is not None:
        out.append(("output.weight", [h, V], spec.type_of("output"), "w"))
    return out


def _filler(spec: ModelSpec, name: str, t: int, n: int, kind: str):
    def fill(dst: np.ndarray) -> None:
        ptr = dst.ctypes.data_as(C.c_void_p)
        if kind == "one":
            if t != T_F32:
                raise ValueError("norm weights are F32")
            _native.gen().gg_fill_f32(ptr, n, 1.0)
            return
        got = _native.gen().gg_random_tensor(t, spec.seed, stream_id(name), n, spec.sigma, ptr)
        if got != dst.size:
            raise RuntimeError(f"{name}: generator wrote {got} bytes, expected {dst.size}")
    return fill


def build_writer(spec: ModelSpec) -> GgufWriter:
    w = GgufWriter()
    arch = spec.arch
    w.add("general.architecture", STR, arch)
    w.add("general.name", STR, f"{spec.name}-seed{spec.seed}")
    w.add(f"{arch}.block_count", U32, spec.n_layers)
    w.add(f"{arch}.embedding_length", U32, spec.hidden)
    w.add(f"{arch}.feed_forward_length", U32, spec.ffn)
    w.add(f"{arch}.attention.head_count", U32, spec.n_heads)
    w.add(f"{arch}.attention.head_count_kv", U32, spec.n_kv)
    w.add(f"{arch}.context_length", U32, spec.ctx)
    w.add(f"{arch}.vocab_size", U32, spec.vocab)
    w.add(f"{arch}.rope.freq_base", F32, float(spec.rope_base))
    w.add(f"{arch}.attention.layer_norm_rms_epsilon", F32, 1e-5 if arch != "gemma2" else 1e-6)
    if spec.head_dim is not None:
        w.add(f"{arch}.attention.key_length", U32, spec.head_dim)
        w.add(f"{arch}.attention.value_length", U32, spec.head_dim)
    if spec.window is not None:
        w.add(f"{arch}.attention.sliding_window", U32, spec.window)
    if spec.attn_softcap is not None:
        w.add(f"{arch}.attn_logit_softcapping", F32, float(spec.attn_softcap))
    if spec.final_softcap is not None:
        w.add(f"{arch}.final_logit_softcapping", F32, float(spec.final_softcap))
    w.add("tokenizer.ggml.model", STR, "gpt2")
    w.add("tokenizer.ggml.tokens", ARR, [f"<t{i}>" for i in range(spec.vocab)], STR)
    w.add("tokenizer.ggml.bos_token_id", U32, spec.bos)
    w.add("tokenizer.ggml.eos_token_id", U32, spec.eos)
    for name, dims, t, kind in tensor_plan(spec):
        n = int(np.prod(dims))
        w.add_tensor(name, dims, t, _filler(spec, name, t, n, kind))
    return w


def build_model(spec: ModelSpec | str, path: str | None = None, threads: int = 0) -> np.ndarray:
    """Returns the whole GGUF image as a uint8 array (and writes it to `path`)."""
    if isinstance(spec, str):
        spec = SPECS[spec]
    _native.gen().gg_set_threads(threads)
    buf = build_writer(spec).build()
    if path:
        buf.tofile(path)
    return buf


def prompt_ids(n: int, vocab: int, seed: int = 0) -> np.ndarray:
    """Uniform random token ids (the benchmark prompts)."""
    out = np.zeros(n, dtype=np.int32)
    _native.gen().gg_uniform_ids(seed, 0x70726F6D7074, n, vocab, out.ctypes.data_as(C.c_void_p))
    return out


def random_blocks(t: int, n_elems: int, seed: int, stream: int, sigma: float = 0.02) -> np.ndarray:
    """Quantized payload of n_elems values (test helper)."""
    nb = _native.gen().gg_tensor_bytes(t, n_elems)
    if nb < 0:
        raise ValueError("bad element count for type")
    out = np.zeros(nb, dtype=np.uint8)
    _native.gen().gg_random_tensor(t, seed, stream, n_elems, sigma, out.ctypes.data_as(C.c_void_p))
    return out


def normal(n: int, seed: int, stream: int, sigma: float = 1.0) -> np.ndarray:
    out = np.zeros(n, dtype=np.float32)
    _native.gen().gg_normal_f32(seed, stream, 0, n, sigma, out.ctypes.data_as(C.c_void_p))
    return out
