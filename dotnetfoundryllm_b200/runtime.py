"""Host-side mirror of the reference's forward-pass seam over the C ABI.

``CudaModel`` is the device counterpart of ``LlamaWeights``/``Gemma2Weights``
(the ``IDisposable modelResources`` of ``LlamaLanguageModel``,
src/DotNetFoundryLLM.Inference/LlamaLanguageModel.cs:48-80) and
``CudaForwardPass`` implements ``IForwardPass``
(src/DotNetFoundryLLM.Architectures/IForwardPass.cs:8-15): ``forward(token_id,
position, kv_cache)`` and ``logits``.  The KV cache lives in HBM; the
``kv_cache`` argument is only the session key, as in the C# backend.

Error behaviour follows the reference: a token id outside [0, vocab) raises
``ArgumentOutOfRangeError`` (LlamaForwardPass.cs:89-93), an unknown tensor type
``NotSupportedError`` (Dequantizer.cs:501-502), a missing tensor
``InvalidOperationError`` (GgufModelLoader.cs:411-412), use after dispose
``ObjectDisposedError`` (LlamaWeights.cs:138-139).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N


class FoundryError(RuntimeError):
    code = -1


class ArgumentError(FoundryError, ValueError):
    """System.ArgumentException."""


class ArgumentOutOfRangeError(ArgumentError, IndexError):
    """System.ArgumentOutOfRangeException."""


class NotSupportedError(FoundryError, NotImplementedError):
    """System.NotSupportedException."""


class InvalidOperationError(FoundryError):
    """System.InvalidOperationException."""


class ObjectDisposedError(InvalidOperationError):
    """System.ObjectDisposedException."""


class DeviceTimeoutError(FoundryError, TimeoutError):
    """A bounded device-side wait expired (FL_ERR_TIMEOUT)."""


class DeviceError(FoundryError):
    """CUDA / NCCL / allocation failure."""


def check(rc: int, what: str = "") -> None:
    if rc == N.FL_OK:
        return
    msg = N.last_error()
    text = f"{what}: {msg}" if what else msg
    if rc == N.FL_ERR_ARG:
        cls = ArgumentOutOfRangeError if ("outside" in msg or "range" in msg) else ArgumentError
    elif rc == N.FL_ERR_UNSUPPORTED:
        cls = NotSupportedError
    elif rc == N.FL_ERR_STATE:
        cls = InvalidOperationError
    elif rc == N.FL_ERR_TIMEOUT:
        cls = DeviceTimeoutError
    else:
        cls = DeviceError
    err = cls(text)
    err.code = rc
    raise err


def _ptr(a: np.ndarray) -> C.c_void_p:
    return a.ctypes.data_as(C.c_void_p)


class CudaModel:
    """Device weights of one model (repacked GGUF blocks, no F32 copy)."""

    def __init__(self, desc: N.FlModelDesc):
        self.lib = N.cuda()
        self.desc = desc
        h = C.c_void_p()
        check(self.lib.fl_model_create(C.byref(desc), C.byref(h)), "fl_model_create")
        self._h = h

    @property
    def handle(self) -> C.c_void_p:
        if self._h is None:
            raise ObjectDisposedError("CudaModel")
        return self._h

    def upload(self, name: str, ggml_type: int, dims: list[int], payload: np.ndarray) -> None:
        payload = np.ascontiguousarray(payload, dtype=np.uint8)
        d = (C.c_uint64 * len(dims))(*dims)
        check(self.lib.fl_model_upload(self.handle, name.encode(), ggml_type, d, len(dims), _ptr(payload),
                                       payload.size), f"upload {name}")

    def finalize(self) -> None:
        check(self.lib.fl_model_finalize(self.handle), "fl_model_finalize")

    def weight_bytes(self) -> float:
        b = C.c_double()
        check(self.lib.fl_model_weight_bytes(self.handle, C.byref(b)))
        return b.value

    def close(self) -> None:
        if self._h is not None:
            self.lib.fl_model_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaForwardPass:
    """IForwardPass over a device session (one KV cache in HBM)."""

    def __init__(self, model: CudaModel, max_ctx: int = 0, max_batch: int = 1):
        self.model = model
        self.lib = model.lib
        self.max_batch = max_batch
        h = C.c_void_p()
        check(self.lib.fl_session_create(model.handle, max_ctx, max_batch, 0, C.byref(h)), "fl_session_create")
        self._h = h
        self.vocab = model.desc.vocab
        self._logits = np.zeros(self.vocab, dtype=np.float32)
        self._argmax = C.c_int32()
        self._kv_key = None

    @property
    def handle(self) -> C.c_void_p:
        if self._h is None:
            raise ObjectDisposedError("CudaForwardPass")
        return self._h

    def prefill(self, tokens, start_pos: int = 0, kv_cache=None) -> None:
        """The prompt path (fl_prefill): K/V of tokens at positions start_pos..
        in one batched pass per layer; follow with forward() for the last
        prompt token."""
        if kv_cache is not self._kv_key or start_pos == 0:
            check(self.lib.fl_session_reset(self.handle, 0))
            self._kv_key = kv_cache
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        check(self.lib.fl_prefill(self.handle, _ptr(t), int(t.size), int(start_pos)), "fl_prefill")

    def time_prefill(self, tokens, start_pos: int = 0, kv_cache=None) -> float:
        """prefill() timed on the device (CUDA events); returns milliseconds."""
        if kv_cache is not self._kv_key or start_pos == 0:
            check(self.lib.fl_session_reset(self.handle, 0))
            self._kv_key = kv_cache
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        ms = C.c_float()
        check(self.lib.fl_time_prefill(self.handle, _ptr(t), int(t.size), int(start_pos), C.byref(ms)),
              "fl_time_prefill")
        return ms.value

    # ── tensor parallelism ──
    def tp_handle(self) -> bytes:
        """This rank's exchange-region handle (FL_TP_HANDLE_BYTES)."""
        buf = (C.c_uint8 * N.FL_TP_HANDLE_BYTES)()
        check(self.lib.fl_session_tp_handle(self.handle, buf), "fl_session_tp_handle")
        return bytes(buf)

    def tp_connect(self, handles: list[bytes]) -> None:
        """Maps every rank's exchange region (handles in rank order)."""
        blob = b"".join(handles)
        if len(blob) != N.FL_TP_HANDLE_BYTES * len(handles):
            raise ArgumentError("each handle is FL_TP_HANDLE_BYTES bytes")
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        check(self.lib.fl_session_tp_connect(self.handle, buf), "fl_session_tp_connect")

    def tp_reset(self) -> None:
        """fl_session_tp_reset: after a tensor-parallel call timed out, every
        rank calls this between two host barriers; the next forward starts a
        new sequence at position 0."""
        check(self.lib.fl_session_tp_reset(self.handle), "fl_session_tp_reset")
        self._kv_key = None

    @property
    def logits(self) -> np.ndarray:
        """IForwardPass.Logits: logits of the most recent forward call."""
        return self._logits

    def forward(self, token_id: int, position: int, kv_cache=None, want_logits: bool = True) -> int:
        """IForwardPass.Forward; returns the greedy argmax as a convenience."""
        if kv_cache is not self._kv_key or position == 0:
            check(self.lib.fl_session_reset(self.handle, 0))
            self._kv_key = kv_cache
        check(self.lib.fl_forward(self.handle, int(token_id), int(position),
                                  _ptr(self._logits) if want_logits else None, C.byref(self._argmax)),
              "fl_forward")
        return int(self._argmax.value)

    def decode_greedy(self, token_id: int, start_pos: int, n_steps: int) -> np.ndarray:
        out = np.zeros(max(n_steps, 1), dtype=np.int32)
        check(self.lib.fl_decode_greedy(self.handle, int(token_id), int(start_pos), int(n_steps), _ptr(out)),
              "fl_decode_greedy")
        return out[:n_steps]

    def topk(self, k: int) -> tuple[np.ndarray, np.ndarray, float]:
        ids = np.zeros(k, dtype=np.int32)
        vals = np.zeros(k, dtype=np.float32)
        thr = C.c_float()
        check(self.lib.fl_topk(self.handle, k, _ptr(ids), _ptr(vals), C.byref(thr)), "fl_topk")
        return ids, vals, thr.value

    def sample(self, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0, repetition_penalty: float = 1.0,
               generated=(), u: float = 0.0) -> int:
        """fl_sample: the GenerateAsync sampling step on the device, on the
        logits of the last forward(); u is the request generator's draw."""
        d = N.FlSamplerDesc(C.sizeof(N.FlSamplerDesc), float(temperature), int(top_k), float(top_p),
                            float(repetition_penalty))
        g = np.ascontiguousarray(generated, dtype=np.int32)
        tok = C.c_int32()
        check(self.lib.fl_sample(self.handle, C.byref(d), _ptr(g) if g.size else None, int(g.size), float(u),
                                 C.byref(tok)), "fl_sample")
        return int(tok.value)

    # ── batched decode (sequence slots) ──
    def reset_slot(self, slot: int) -> None:
        check(self.lib.fl_session_reset(self.handle, int(slot)), "fl_session_reset")

    def prefill_seq(self, slot: int, tokens, start_pos: int = 0) -> None:
        """fl_prefill_seq: the prompt path into sequence slot `slot`."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        check(self.lib.fl_prefill_seq(self.handle, int(slot), _ptr(t), int(t.size), int(start_pos)),
              "fl_prefill_seq")

    def forward_batch(self, tokens, positions, slots, want_logits: bool = False):
        """fl_forward_batch: one step of len(tokens) sequences; returns the
        argmax per row and, if asked, the [rows x vocab] logits."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(positions, dtype=np.int32)
        sl = np.ascontiguousarray(slots, dtype=np.int32)
        am = np.zeros(t.size, dtype=np.int32)
        lg = np.zeros((t.size, self.vocab), dtype=np.float32) if want_logits else None
        check(self.lib.fl_forward_batch(self.handle, int(t.size), _ptr(t), _ptr(p), _ptr(sl),
                                        _ptr(lg) if want_logits else None, _ptr(am)), "fl_forward_batch")
        return (am, lg) if want_logits else am

    def time_decode(self, token_id: int, start_pos: int, n_steps: int) -> float:
        ms = C.c_float()
        check(self.lib.fl_time_decode(self.handle, int(token_id), int(start_pos), int(n_steps), C.byref(ms)),
              "fl_time_decode")
        return ms.value

    def profile_step(self, token_id: int, position: int) -> dict:
        ms = (C.c_double * N.FL_PROF_N)()
        by = (C.c_double * N.FL_PROF_N)()
        nl = C.c_int32()
        check(self.lib.fl_profile_step(self.handle, int(token_id), int(position), ms, by, C.byref(nl)),
              "fl_profile_step")
        names = ["matvec", "attention", "other", "step"]
        return {"ms": dict(zip(names, list(ms))), "bytes": dict(zip(names, list(by))), "launches": nl.value}

    def launches_per_step(self) -> int:
        n = C.c_int32()
        check(self.lib.fl_session_launches_per_step(self.handle, C.byref(n)))
        return n.value

    def close(self) -> None:
        if self._h is not None:
            self.lib.fl_session_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def generate_greedy(fwd: CudaForwardPass, prompt: np.ndarray, max_tokens: int, eos: int | None = None,
                    collect_logits: bool = False):
    """LlamaLanguageModel.GenerateAsync with Temperature = 0
    (LlamaLanguageModel.cs:126-293): Forward every prompt token but the last,
    then forward the last prompt token as decode step 0 and feed back the
    ArgMax; stop at EOS or after max_tokens.  Returns (tokens, logits|None)."""
    kv = object()
    pos = 0
    for i in range(len(prompt) - 1):
        fwd.forward(int(prompt[i]), pos, kv, want_logits=False)
        pos += 1
    nxt = int(prompt[-1]) if len(prompt) else fwd.model.desc.bos
    toks, logs = [], []
    for _ in range(max_tokens):
        nxt = fwd.forward(nxt, pos, kv, want_logits=collect_logits)
        pos += 1
        if collect_logits:
            logs.append(fwd.logits.copy())
        toks.append(nxt)
        if eos is not None and nxt == eos:
            break
    return np.array(toks, dtype=np.int32), (np.stack(logs) if collect_logits else None)


class XoshiroRandom:
    """Core/XoshiroRandom.cs: xoshiro256** seeded by four SplitMix64 outputs
    (XoshiroRandom.cs:9-25); NextFloat rounds the top 53 bits, as a double in
    [0, 1), to float (:44)."""

    M = (1 << 64) - 1

    def __init__(self, seed: int):
        x = seed & self.M
        self.s = []
        for _ in range(4):
            x = (x + 0x9E3779B97F4A7C15) & self.M
            z = x
            z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & self.M
            z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & self.M
            self.s.append(z ^ (z >> 31))

    @staticmethod
    def _rotl(x: int, k: int) -> int:
        return ((x << k) | (x >> (64 - k))) & XoshiroRandom.M

    def next_uint64(self) -> int:
        s0, s1, s2, s3 = self.s
        result = (self._rotl((s1 * 5) & self.M, 7) * 9) & self.M
        t = (s1 << 17) & self.M
        s2 ^= s0
        s3 ^= s1
        s1 ^= s2
        s0 ^= s3
        s2 ^= t
        s3 = self._rotl(s3, 45)
        self.s = [s0, s1, s2, s3]
        return result

    def next_float(self) -> float:
        return float(np.float32((self.next_uint64() >> 11) * (1.0 / (1 << 53))))


def generate(fwd: CudaForwardPass, prompt: np.ndarray, max_tokens: int, temperature: float = 1.0, top_k: int = 0,
             top_p: float = 1.0, seed: int = 0, repetition_penalty: float = 1.0, eos: int | None = None) -> np.ndarray:
    """LlamaLanguageModel.GenerateAsync with a SamplerPipeline
    (LlamaLanguageModel.cs:126-293, 343-373): the prompt as in
    generate_greedy, then every step forward → repetition penalty over the
    tokens generated so far → SamplerPipeline.Sample, all on the device; the
    only per-step host work is the generator draw."""
    import time
    rng = XoshiroRandom(seed if seed else time.monotonic_ns())
    kv = object()
    pos = 0
    for i in range(len(prompt) - 1):
        fwd.forward(int(prompt[i]), pos, kv, want_logits=False)
        pos += 1
    nxt = int(prompt[-1]) if len(prompt) else fwd.model.desc.bos
    toks: list[int] = []
    for _ in range(max_tokens):
        fwd.forward(nxt, pos, kv, want_logits=False)
        pos += 1
        u = rng.next_float() if temperature != 0.0 else 0.0
        nxt = fwd.sample(temperature, top_k, top_p, repetition_penalty, toks, u)
        toks.append(nxt)
        if eos is not None and nxt == eos:
            break
    return np.array(toks, dtype=np.int32)


def generate_batch_greedy(fwd: CudaForwardPass, prompts, max_tokens: int) -> list[np.ndarray]:
    """Greedy completion of several prompts at once, one sequence slot each:
    every prompt but its last token through the prompt path, then batched
    decode steps (each row the loop of LlamaLanguageModel.GenerateAsync with
    Temperature = 0)."""
    B = len(prompts)
    if B > fwd.max_batch:
        raise ArgumentError(f"{B} prompts for {fwd.max_batch} sequence slots")
    pos = np.zeros(B, dtype=np.int32)
    nxt = np.zeros(B, dtype=np.int32)
    for b, pr in enumerate(prompts):
        fwd.reset_slot(b)
        fwd.prefill_seq(b, pr[:-1], 0)
        pos[b] = len(pr) - 1
        nxt[b] = int(pr[-1])
    out = np.zeros((B, max_tokens), dtype=np.int32)
    slots = np.arange(B, dtype=np.int32)
    for step in range(max_tokens):
        nxt = fwd.forward_batch(nxt, pos, slots)
        out[:, step] = nxt
        pos += 1
    return [out[b] for b in range(B)]


def dequantize(ggml_type: int, raw: np.ndarray, dst_len: int | None = None) -> np.ndarray:
    """Dequantizer.Dequantize on the device (bit-exact)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    lib = N.cuda()
    if dst_len is None:
        from .gguf import BLOCK
        be, bb = BLOCK.get(ggml_type, (1, 1))
        dst_len = raw.size // bb * be
    out = np.zeros(max(dst_len, 1), dtype=np.float32)
    check(lib.fl_dequant(ggml_type, _ptr(raw), raw.size, _ptr(out), dst_len), "fl_dequant")
    return out[:dst_len]


def matvec(ggml_type: int, raw: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    """One dequant-matvec launch through the forward pass's kernel."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, dtype=np.float32)
    check(N.cuda().fl_matvec(ggml_type, _ptr(raw), raw.size, rows, cols, _ptr(x), _ptr(y)), "fl_matvec")
    return y


def gemm_f16(a: np.ndarray, b: np.ndarray, m: int, n: int, k: int, alpha: float = 1.0, beta: float = 0.0,
             y: np.ndarray | None = None, batch: int = 1, a_batch_rows: int = 0, b_batch_rows: int = 0,
             ksplit: int = 1, causal: int = 0, c_grp: int = 1, c_start: int = 0, c_seg: int = 0) -> np.ndarray:
    """fl_gemm_f16: y[b][j][i] = alpha * a[b][i] . b[b][j] (+ beta * y) on the
    tensor cores for i < m, j < n over k; a and b are float16 arrays whose
    last axis is the row stride (k of it used).  ksplit / causal as the C
    hook documents."""
    a = np.ascontiguousarray(a, dtype=np.float16)
    b = np.ascontiguousarray(b, dtype=np.float16)
    y = np.zeros((batch, n, m), np.float32) if y is None else np.ascontiguousarray(y, dtype=np.float32).copy()
    check(N.cuda().fl_gemm_f16(_ptr(a), a.shape[-1], _ptr(b), b.shape[-1], m, n, k, batch, a_batch_rows,
                               b_batch_rows, alpha, beta, ksplit, causal, c_grp, c_start, c_seg, _ptr(y)),
          "fl_gemm_f16")
    return y


def init_tensor_parallel(tp: int, devices: list[int] | None = None) -> None:
    """fl_init: the devices of the process's tensor-parallel groups (models
    loaded with tp_rank=FL_TP_ALL, tp_size=tp); None = devices 0..tp-1."""
    arr = (C.c_int32 * tp)(*devices) if devices is not None else None
    if devices is not None and len(devices) != tp:
        raise ArgumentError(f"{len(devices)} devices for {tp} ranks")
    check(N.cuda().fl_init(tp, arr), "fl_init")


def connect_tensor_parallel(fwd, all_gather) -> None:
    """Connects one rank's session to its peers: `all_gather(bytes)` must return
    every rank's bytes in rank order (a torch.distributed gather, a file, ...)."""
    handles = list(all_gather(fwd.tp_handle()))
    fwd.tp_connect(handles)
