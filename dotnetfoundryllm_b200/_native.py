"""ctypes bindings of the in-tree native libraries.

``cuda()`` loads ``_lib/libfoundry_cuda.so`` (the C ABI of
``include/foundry_cuda.h``); ``gen()`` loads ``_lib/libfoundry_gen.so`` (the
synthetic weight generator).  Both raise if the library is missing: there is
no fallback path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "_lib"

FL_OK = 0
FL_ERR_ARG = 1
FL_ERR_OOM = 2
FL_ERR_CUDA = 3
FL_ERR_NCCL = 4
FL_ERR_TIMEOUT = 5
FL_ERR_UNSUPPORTED = 6
FL_ERR_STATE = 7

FL_ARCH_LLAMA, FL_ARCH_MISTRAL, FL_ARCH_GEMMA2, FL_ARCH_QWEN2 = 0, 1, 2, 3

FL_PROF_MATVEC, FL_PROF_ATTN, FL_PROF_OTHER, FL_PROF_STEP, FL_PROF_N = 0, 1, 2, 3, 4

FL_TOPK_DEVICE_MAX_N = 262144
FL_TP_HANDLE_BYTES = 64
FL_TP_ALL = -1  # fl_model_desc.tp_rank of a group driven from one thread


class FlModelDesc(C.Structure):
    _fields_ = [
        ("struct_size", C.c_int32),
        ("arch", C.c_int32),
        ("n_layers", C.c_int32),
        ("hidden", C.c_int32),
        ("ffn", C.c_int32),
        ("n_heads", C.c_int32),
        ("n_kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("vocab", C.c_int32),
        ("max_ctx", C.c_int32),
        ("bos", C.c_int32),
        ("eos", C.c_int32),
        ("sliding_window", C.c_int32),
        ("rope_scaled", C.c_int32),
        ("rms_eps", C.c_float),
        ("rope_base", C.c_float),
        ("rope_factor", C.c_float),
        ("attn_softcap", C.c_float),
        ("final_softcap", C.c_float),
        ("attn_scale", C.c_float),
        ("device", C.c_int32),
        ("tp_rank", C.c_int32),
        ("tp_size", C.c_int32),
        ("nccl_id", C.c_void_p),
    ]


class FlMatrixLayout(C.Structure):
    _fields_ = [
        ("ggml_type", C.c_int32),
        ("fmt", C.c_int32),
        ("expanded", C.c_int32),
        ("rows", C.c_int32),
        ("cols", C.c_int32),
        ("n_tiles", C.c_int32),
        ("n_kb", C.c_int32),
        ("unit_bytes", C.c_int32),
        ("hdr_bytes", C.c_int32),
        ("total_bytes", C.c_int64),
        ("gguf_bytes", C.c_int64),
    ]


class FlSamplerDesc(C.Structure):
    _fields_ = [
        ("struct_size", C.c_int32),
        ("temperature", C.c_float),
        ("top_k", C.c_int32),
        ("top_p", C.c_float),
        ("repetition_penalty", C.c_float),
    ]


# Every entry point declared in include/foundry_cuda.h: (name, restype, argtypes)
PUBLIC_API = [
    ("fl_last_error", C.c_char_p, []),
    ("fl_abi_version", C.c_int32, []),
    ("fl_model_create", C.c_int, [C.POINTER(FlModelDesc), C.POINTER(C.c_void_p)]),
    ("fl_model_upload", C.c_int, [C.c_void_p, C.c_char_p, C.c_int32, C.POINTER(C.c_uint64), C.c_int32,
                                  C.c_void_p, C.c_uint64]),
    ("fl_model_finalize", C.c_int, [C.c_void_p]),
    ("fl_model_destroy", None, [C.c_void_p]),
    ("fl_session_create", C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_void_p)]),
    ("fl_session_reset", C.c_int, [C.c_void_p, C.c_int32]),
    ("fl_forward", C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
    ("fl_decode_greedy", C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p]),
    ("fl_prefill", C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32]),
    ("fl_prefill_seq", C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_int32]),
    ("fl_forward_batch", C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_void_p]),
    ("fl_topk", C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("fl_topk_device", C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("fl_sample", C.c_int, [C.c_void_p, C.POINTER(FlSamplerDesc), C.c_void_p, C.c_int32, C.c_float,
                            C.POINTER(C.c_int32)]),
    ("fl_session_tp_handle", C.c_int, [C.c_void_p, C.c_void_p]),
    ("fl_session_tp_connect", C.c_int, [C.c_void_p, C.c_void_p]),
    ("fl_session_tp_reset", C.c_int, [C.c_void_p]),
    ("fl_init", C.c_int, [C.c_int32, C.POINTER(C.c_int32)]),
    ("fl_session_destroy", None, [C.c_void_p]),
    ("fl_dequant", C.c_int, [C.c_int32, C.c_void_p, C.c_uint64, C.c_void_p, C.c_uint64]),
    ("fl_matvec", C.c_int, [C.c_int32, C.c_void_p, C.c_uint64, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
    ("fl_gemm_f16", C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_int32,
                              C.c_int32, C.c_int32, C.c_int32, C.c_float, C.c_float, C.c_int32, C.c_int32,
                              C.c_int32, C.c_int32, C.c_int32, C.c_void_p]),
    ("fl_profile_step", C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("fl_time_decode", C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_float)]),
    ("fl_time_prefill", C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.POINTER(C.c_float)]),
    ("fl_model_weight_bytes", C.c_int, [C.c_void_p, C.POINTER(C.c_double)]),
    ("fl_session_launches_per_step", C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
]

INTERNAL_API = [
    ("fl_layout_for", C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.POINTER(FlMatrixLayout)]),
    ("fl_repack", C.c_int, [C.POINTER(FlMatrixLayout), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]),
    ("fl_emulate_matvec", C.c_int, [C.POINTER(FlMatrixLayout), C.c_void_p, C.c_void_p, C.c_void_p]),
    ("fl_session_phase_ms", C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.POINTER(C.c_int32)]),
    ("fl_session_cta_done_ms", C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.POINTER(C.c_int32)]),
    ("fl_session_detail", C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    ("fl_dequant_split_test", C.c_int, [C.c_int32, C.c_void_p, C.c_uint64, C.c_int32, C.c_int32, C.c_void_p]),
    ("fl_tp_slice", C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
]

GEN_API = [
    ("gg_set_threads", C.c_int, [C.c_int]),
    ("gg_normal_f32", None, [C.c_uint64, C.c_uint64, C.c_int64, C.c_int64, C.c_float, C.c_void_p]),
    ("gg_uniform_ids", None, [C.c_uint64, C.c_uint64, C.c_int64, C.c_int32, C.c_void_p]),
    ("gg_tensor_bytes", C.c_int64, [C.c_int, C.c_int64]),
    ("gg_quantize", C.c_int64, [C.c_int, C.c_void_p, C.c_int64, C.c_void_p]),
    ("gg_random_tensor", C.c_int64, [C.c_int, C.c_uint64, C.c_uint64, C.c_int64, C.c_float, C.c_void_p]),
    ("gg_fill_f32", None, [C.c_void_p, C.c_int64, C.c_float]),
    ("gg_f32_to_f16", C.c_uint16, [C.c_float]),
    ("gg_f16_to_f32", C.c_float, [C.c_uint16]),
]

_cuda = None
_gen = None


def _load(path: Path, api) -> C.CDLL:
    if not path.exists():
        raise RuntimeError(f"native library {path} is missing: run `python -m dotnetfoundryllm_b200.build`")
    lib = C.CDLL(str(path))
    for name, res, args in api:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def cuda() -> C.CDLL:
    global _cuda
    if _cuda is None:
        _cuda = _load(LIB_DIR / "libfoundry_cuda.so", PUBLIC_API + INTERNAL_API)
    return _cuda


def gen() -> C.CDLL:
    global _gen
    if _gen is None:
        _gen = _load(LIB_DIR / "libfoundry_gen.so", GEN_API)
    return _gen


def last_error() -> str:
    msg = cuda().fl_last_error()
    return msg.decode("utf-8", "replace") if msg else ""
