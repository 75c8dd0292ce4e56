"""ctypes wrapper of the CPU restatement (``oracle/_build/libfl_oracle.so``).

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path and the timed
CPU baseline.  Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU
baseline import this module; the product package never does.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libfl_oracle.so"

OK, ARGUMENT_EXCEPTION, NOT_SUPPORTED, ARGUMENT_OUT_OF_RANGE, INVALID_OPERATION, MODEL_LOAD = 0, -1, -2, -3, -4, -5

_lib = None


def build() -> Path:
    src = [HERE / "fl_oracle.c", HERE / "fl_oracle.h", HERE / "Makefile"]
    if not LIB.exists() or any(s.stat().st_mtime > LIB.stat().st_mtime for s in src):
        subprocess.run(["make", "-C", str(HERE)], check=True, capture_output=True)
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = C.CDLL(str(LIB))
        vp, i32, i64, f32 = C.c_void_p, C.c_int, C.c_int64, C.c_float
        sig = {
            "or_half_to_float": (f32, [C.c_uint16]),
            "or_bf16_to_float": (f32, [C.c_uint16]),
            "or_element_count": (i64, [i32, i64]),
            "or_dequantize": (i32, [i32, vp, i64, vp, i64]),
            "or_dot": (f32, [vp, vp, i32]),
            "or_rmsnorm": (None, [vp, vp, vp, i32, f32]),
            "or_gemma_rmsnorm": (None, [vp, vp, vp, i32]),
            "or_softmax": (None, [vp, i32]),
            "or_silu": (None, [vp, i32]),
            "or_gelu": (None, [vp, i32]),
            "or_softcap": (None, [vp, i32, f32]),
            "or_argmax": (i32, [vp, i32]),
            "or_apply_topk": (None, [vp, i32, i32]),
            "or_rope": (None, [vp, f32, vp, i32]),
            "or_xoshiro_seed": (None, [C.c_uint64, vp]),
            "or_xoshiro_next": (C.c_uint64, [vp]),
            "or_xoshiro_next_float": (f32, [vp]),
            "or_apply_repetition_penalty": (None, [vp, i32, vp, i32, f32]),
            "or_apply_topp": (None, [vp, i32, f32]),
            "or_sample_from_probs": (i32, [vp, i32, f32]),
            "or_sampler_pipeline": (i32, [vp, i32, f32, i32, f32, f32]),
            "or_gguf_parse": (vp, [vp, i64, C.c_char_p, i32]),
            "or_gguf_free": (None, [vp]),
            "or_gguf_version": (C.c_uint32, [vp]),
            "or_gguf_tensor_count": (i64, [vp]),
            "or_gguf_kv_count": (i64, [vp]),
            "or_gguf_data_start": (i64, [vp]),
            "or_gguf_find_tensor": (i64, [vp, C.c_char_p]),
            "or_gguf_tensor_info": (i32, [vp, i64, vp, vp, vp, vp, vp]),
            "or_model_load_ex": (vp, [vp, i64, i32, i32, C.c_char_p, i32]),
            "or_model_load": (vp, [vp, i64, i32, C.c_char_p, i32]),
            "or_model_free": (None, [vp]),
            "or_model_config": (None, [vp, vp, vp, vp]),
            "or_session_create": (vp, [vp]),
            "or_session_free": (None, [vp]),
            "or_session_length": (i32, [vp]),
            "or_session_fake_length": (i32, [vp, i32]),
            "or_forward": (i32, [vp, i32, i32, vp]),
            "or_forward_layers": (i32, [vp, i32, i32, i32]),
            "or_forward_head": (i32, [vp, vp]),
            "or_generate_greedy": (i32, [vp, vp, i32, i32, vp, vp]),
            "or_set_threads": (None, [i32]),
            "or_get_threads": (i32, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray) -> C.c_void_p:
    return a.ctypes.data_as(C.c_void_p)


def dequantize(t: int, raw: np.ndarray, dst_len: int | None = None) -> tuple[int, np.ndarray]:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    if dst_len is None:
        n = lib().or_element_count(t, raw.size)
        dst_len = max(int(n), 0)
    out = np.zeros(max(dst_len, 1), dtype=np.float32)
    rc = lib().or_dequantize(t, _p(raw), raw.size, _p(out), dst_len)
    return rc, out[:dst_len]


def matvec(t: int, raw: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    """LinearProjection over the dequantized F32 matrix (the reference path)."""
    rc, w = dequantize(t, raw, rows * cols)
    assert rc == OK, rc
    w = w.reshape(rows, cols)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, dtype=np.float32)
    L = lib()
    for r in range(rows):
        y[r] = L.or_dot(_p(x), _p(np.ascontiguousarray(w[r])), cols)
    return y


class Model:
    """``lazy=True`` keeps the weight matrices as the image's quantized blocks
    and dequantizes each row where it is used (the same floats, so the same
    results): host memory stays at the size of the file instead of F32."""

    def __init__(self, image: np.ndarray, max_layers: int = -1, lazy: bool = False):
        self.image = np.ascontiguousarray(image, dtype=np.uint8)
        err = C.create_string_buffer(512)
        self.h = lib().or_model_load_ex(_p(self.image), self.image.size, max_layers, int(lazy), err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())
        arch = C.c_int()
        iv = (C.c_int * 12)()
        fv = (C.c_float * 8)()
        lib().or_model_config(self.h, C.byref(arch), iv, fv)
        self.arch = arch.value
        (self.n_layers, self.hidden, self.ffn, self.n_heads, self.n_kv, self.head_dim, self.vocab, self.max_ctx,
         self.bos, self.eos, self.window, self.rope_scaled) = list(iv)
        self.rope_base, self.rope_factor, self.attn_softcap, self.final_softcap, self.attn_scale = list(fv)[:5]

    def close(self):
        if self.h:
            lib().or_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def generate_greedy(self, prompt: np.ndarray, max_tokens: int, collect_logits: bool = False):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        toks = np.zeros(max_tokens, dtype=np.int32)
        logs = np.zeros((max_tokens, self.vocab), dtype=np.float32) if collect_logits else None
        n = lib().or_generate_greedy(self.h, _p(prompt), prompt.size, max_tokens, _p(toks),
                                     _p(logs) if collect_logits else None)
        if n < 0:
            raise RuntimeError(f"oracle error {n}")
        return toks[:n], (logs[:n] if collect_logits else None)


class Session:
    def __init__(self, model: Model):
        self.model = model
        self.h = lib().or_session_create(model.h)
        self.logits = np.zeros(model.vocab, dtype=np.float32)

    def forward(self, token: int, position: int) -> int:
        return lib().or_forward(self.h, token, position, _p(self.logits))

    def forward_layers(self, token: int, position: int, n_layers: int) -> int:
        return lib().or_forward_layers(self.h, token, position, n_layers)

    def fake_length(self, n: int) -> int:
        return lib().or_session_fake_length(self.h, n)

    def forward_head(self) -> int:
        return lib().or_forward_head(self.h, _p(self.logits))

    def close(self):
        if self.h:
            lib().or_session_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def set_threads(n: int) -> None:
    lib().or_set_threads(n)


class Xoshiro:
    """XoshiroRandom (Core/XoshiroRandom.cs) through the C restatement."""

    def __init__(self, seed: int):
        self.state = np.zeros(4, dtype=np.uint64)
        lib().or_xoshiro_seed(C.c_uint64(seed), _p(self.state))

    def next_uint64(self) -> int:
        return int(lib().or_xoshiro_next(_p(self.state)))

    def next_float(self) -> float:
        return float(lib().or_xoshiro_next_float(_p(self.state)))


def apply_repetition_penalty(logits: np.ndarray, generated, penalty: float) -> np.ndarray:
    out = np.ascontiguousarray(logits, dtype=np.float32).copy()
    g = np.ascontiguousarray(generated, dtype=np.int32)
    lib().or_apply_repetition_penalty(_p(out), out.size, _p(g), g.size, penalty)
    return out


def apply_topp(probs: np.ndarray, p: float) -> np.ndarray:
    out = np.ascontiguousarray(probs, dtype=np.float32).copy()
    lib().or_apply_topp(_p(out), out.size, p)
    return out


def sampler_pipeline(logits: np.ndarray, temperature: float, top_k: int, top_p: float, u: float) -> tuple[int, np.ndarray]:
    """SamplerPipeline.Sample; returns the token and the final distribution
    (the transformed logits array)."""
    out = np.ascontiguousarray(logits, dtype=np.float32).copy()
    tok = lib().or_sampler_pipeline(_p(out), out.size, temperature, top_k, top_p, u)
    return int(tok), out
