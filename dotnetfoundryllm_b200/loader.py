"""GGUF → device model: the host half of ``GgufModelLoader`` for the CUDA
backend.

``build_desc`` restates ``GgufModelLoader.Build`` / ``BuildConfig`` /
``BuildMistral`` / ``BuildGemma2`` (src/DotNetFoundryLLM.ModelFormats.Gguf/
GgufModelLoader.cs:89-334): the same metadata keys, defaults and integer
truncation.  ``load`` then hands every tensor's RAW block bytes to
``fl_model_upload`` — the replacement for ``LoadTensor``'s F32 expansion
(:409-418).
"""
from __future__ import annotations

import math

import numpy as np

from . import _native as N
from .gguf import GgufFile, parse
from .runtime import CudaModel, NotSupportedError

INT32_MAX = 2147483647

ARCHS = {"llama": N.FL_ARCH_LLAMA, "llama3": N.FL_ARCH_LLAMA, "llama4": N.FL_ARCH_LLAMA,
         "mistral": N.FL_ARCH_MISTRAL, "gemma": N.FL_ARCH_GEMMA2, "gemma2": N.FL_ARCH_GEMMA2,
         "qwen2": N.FL_ARCH_QWEN2}


def _i32(v: int) -> int:
    """C# (int) of a ulong: keep the low 32 bits, signed."""
    v &= 0xFFFFFFFF
    return v - (1 << 32) if v >= (1 << 31) else v


def build_desc(g: GgufFile, device: int = 0, max_ctx: int | None = None, tp_rank: int = 0,
               tp_size: int = 1) -> N.FlModelDesc:
    arch = g.get_string("general.architecture", "llama")
    if arch not in ARCHS:
        raise NotSupportedError(f"Architecture '{arch}' is not supported. Supported: llama, mistral, gemma2, qwen2.")
    code = ARCHS[arch]
    p = arch
    if code == N.FL_ARCH_GEMMA2:
        p = "gemma2" if "gemma2.block_count" in g.metadata else "gemma"
    d = N.FlModelDesc()
    d.struct_size = N.C.sizeof(N.FlModelDesc)
    d.arch = code
    d.n_layers = _i32(g.get_uint(f"{p}.block_count"))
    d.hidden = _i32(g.get_uint(f"{p}.embedding_length"))
    d.ffn = _i32(g.get_uint(f"{p}.feed_forward_length"))
    hc = g.get_uint(f"{p}.attention.head_count")
    d.n_heads = _i32(hc)
    d.n_kv_heads = _i32(g.get_uint(f"{p}.attention.head_count_kv", hc))
    d.max_ctx = _i32(g.get_uint(f"{p}.context_length", 4096))
    if max_ctx is not None:
        d.max_ctx = min(d.max_ctx, max_ctx)
    d.vocab = _i32(g.get_uint(f"{p}.vocab_size", g.get_uint("tokenizer.ggml.tokens", 32000, array_length=True)))
    d.rope_base = g.get_float(f"{p}.rope.freq_base", 10000.0)
    d.rope_factor = g.get_float(f"{p}.rope.scaling.factor", g.get_float(f"{p}.rope.freq_scale", 1.0))
    rtype = g.get_string(f"{p}.rope.scaling.type", "none").lower()
    d.rope_scaled = 1 if rtype in ("linear", "yarn") and d.rope_factor > 0 else 0
    d.bos = _i32(g.get_uint("tokenizer.ggml.bos_token_id", 1))
    d.eos = _i32(g.get_uint("tokenizer.ggml.eos_token_id", 2))
    d.head_dim = d.hidden // d.n_heads if d.n_heads else 0
    d.sliding_window = INT32_MAX
    d.rms_eps = 1e-5  # TensorOperations.RmsNorm default; the loader never passes the GGUF epsilon
    d.attn_scale = 1.0 / math.sqrt(d.head_dim) if d.head_dim else 0.0
    if code == N.FL_ARCH_MISTRAL:
        d.sliding_window = _i32(g.get_uint("mistral.attention.sliding_window", INT32_MAX))
    if code == N.FL_ARCH_GEMMA2:
        hdo = _i32(g.get_uint(f"{p}.attention.key_length", 0))
        if hdo > 0:
            d.head_dim = hdo
        d.sliding_window = _i32(g.get_uint(f"{p}.attention.sliding_window", INT32_MAX))
        d.attn_softcap = g.get_float(f"{p}.attn_logit_softcapping", 0.0)
        d.final_softcap = g.get_float(f"{p}.final_logit_softcapping", 0.0)
        d.attn_scale = g.get_float(f"{p}.attention.query_pre_attn_scalar",
                                   float(np.float32(1.0) / np.sqrt(np.float32(d.head_dim))))
        d.rms_eps = 1e-6
    else:
        d.attn_scale = float(np.float32(1.0) / np.sqrt(np.float32(d.head_dim)))
    d.device = device
    d.tp_rank, d.tp_size = tp_rank, tp_size
    d.nccl_id = None
    return d


def load(gguf_image, device: int = 0, max_ctx: int | None = None, tp_rank: int = 0, tp_size: int = 1) -> CudaModel:
    """Parses a GGUF image (bytes / numpy / memmap) and uploads it (this rank's
    shard when tp_size > 1: the shim slices the raw blocks).  tp_rank
    FL_TP_ALL (-1) makes a group of tp_size ranks on the devices `fl_init`
    chose (runtime.init_tensor_parallel), driven from the calling thread."""
    g = gguf_image if isinstance(gguf_image, GgufFile) else parse(gguf_image)
    desc = build_desc(g, device, max_ctx, tp_rank, tp_size)
    model = CudaModel(desc)
    try:
        for t in g.tensors:
            model.upload(t.name, t.type, t.dims, g.tensor_bytes(t))
        model.finalize()
    except Exception:
        model.close()
        raise
    return model
