"""The C ABI without a GPU: the library loads, exports every entry point that
include/foundry_cuda.h declares, and rejects bad arguments the way the
reference does before any device work (Dequantizer.Dequantize's
ArgumentException / NotSupportedException, LlamaForwardPass's head-config
check)."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from dotnetfoundryllm_b200 import _native as N
from dotnetfoundryllm_b200 import loader
from dotnetfoundryllm_b200.runtime import ArgumentError, NotSupportedError, check

HEADER = Path(__file__).resolve().parents[1] / "include" / "foundry_cuda.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fl_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_the_abi():
    names = declared_functions()
    for must in ("fl_model_create", "fl_model_upload", "fl_session_create", "fl_forward", "fl_dequant",
                 "fl_last_error", "fl_topk", "fl_decode_greedy"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(str(N.LIB_DIR / "libfoundry_cuda.so"))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert missing == []


def test_python_binding_covers_header():
    bound = {name for name, _, _ in N.PUBLIC_API}
    assert set(declared_functions()) <= bound


def test_abi_version():
    assert N.cuda().fl_abi_version() == 1


def test_desc_struct_layout_matches_header():
    # int32 x 14, float x 6, int32 x 3, pointer
    assert C.sizeof(N.FlModelDesc) == 14 * 4 + 6 * 4 + 3 * 4 + 4 + 8


@pytest.mark.parametrize("t,n,dst,code", [
    (99, 4, 1, N.FL_ERR_UNSUPPORTED),   # Dequantize_UnknownType_Throws
    (0, 5, 1, N.FL_ERR_ARG),            # DequantizeF32_WrongLength_Throws
    (2, 17, 32, N.FL_ERR_ARG),          # DequantizeQ4_0_WrongLength_Throws
    (8, 33, 32, N.FL_ERR_ARG),          # DequantizeQ8_0_WrongLength_Throws
    (12, 143, 256, N.FL_ERR_ARG),       # DequantizeQ4_K_WrongLength_Throws
    (13, 175, 256, N.FL_ERR_ARG),       # DequantizeQ5_K_WrongLength_Throws
    (12, 144, 255, N.FL_ERR_ARG),       # destination too small
])
def test_dequant_argument_errors_without_device(t, n, dst, code):
    src = np.zeros(n, np.uint8)
    out = np.zeros(max(dst, 1), np.float32)
    rc = N.cuda().fl_dequant(t, src.ctypes.data_as(C.c_void_p), n, out.ctypes.data_as(C.c_void_p), dst)
    assert rc == code
    assert N.last_error() != ""
    with pytest.raises(NotSupportedError if code == N.FL_ERR_UNSUPPORTED else ArgumentError):
        check(rc)


def test_model_create_rejects_bad_heads():
    d = N.FlModelDesc()
    d.struct_size = C.sizeof(N.FlModelDesc)
    d.arch, d.n_layers, d.hidden, d.ffn, d.n_heads, d.n_kv_heads = 0, 1, 512, 1408, 8, 3
    d.head_dim, d.vocab, d.max_ctx = 64, 32000, 64
    h = C.c_void_p()
    assert N.cuda().fl_model_create(C.byref(d), C.byref(h)) == N.FL_ERR_ARG
    assert "Invalid attention head configuration" in N.last_error()
    d.struct_size = 4
    assert N.cuda().fl_model_create(C.byref(d), C.byref(h)) == N.FL_ERR_ARG


def test_loader_desc_matches_oracle_config():
    from oracle import oracle as O
    from conftest import model_image
    for name in ("tiny", "tiny-mistral", "tiny-gemma2"):
        img = model_image(name)
        from dotnetfoundryllm_b200 import gguf
        d = loader.build_desc(gguf.parse(img))
        m = O.Model(img, max_layers=0)
        assert (d.arch, d.n_layers, d.hidden, d.ffn, d.n_heads, d.n_kv_heads, d.head_dim, d.vocab, d.max_ctx,
                d.bos, d.eos, d.sliding_window) == (m.arch, m.n_layers, m.hidden, m.ffn, m.n_heads, m.n_kv,
                                                    m.head_dim, m.vocab, m.max_ctx, m.bos, m.eos, m.window)
        assert np.float32(d.attn_scale) == np.float32(m.attn_scale)
        assert np.float32(d.rope_base) == np.float32(m.rope_base)
        assert np.float32(d.attn_softcap) == np.float32(m.attn_softcap)
        assert np.float32(d.final_softcap) == np.float32(m.final_softcap)
        m.close()


def _zero(t):
    if t in (C.c_int32, C.c_uint64, C.c_int64, C.c_int):
        return 0
    if t is C.c_float:
        return 0.0
    return None


@pytest.mark.parametrize("name,args", [(n, a) for n, r, a in N.PUBLIC_API
                                       if r is C.c_int and n not in ("fl_dequant", "fl_init")])
def test_entry_points_reject_null_arguments_before_device_work(name, args):
    """Every entry point that returns a status refuses null handles/pointers
    with FL_ERR_ARG and a message (the reference's ArgumentNullException)."""
    rc = getattr(N.cuda(), name)(*[_zero(t) for t in args])
    assert rc == N.FL_ERR_ARG, (name, rc)
    assert N.last_error() != ""


def test_destroy_of_null_handles_is_a_no_op():
    N.cuda().fl_model_destroy(None)
    N.cuda().fl_session_destroy(None)


def test_init_and_group_checks_before_device_work():
    """fl_init refuses rank counts other than 1, 2, 4, 8 and shared or negative
    devices before any device call; a group model needs 2, 4 or 8 ranks."""
    lib = N.cuda()
    assert lib.fl_init(3, None) == N.FL_ERR_UNSUPPORTED
    assert lib.fl_init(0, None) == N.FL_ERR_UNSUPPORTED
    assert lib.fl_init(2, (C.c_int32 * 2)(0, 0)) == N.FL_ERR_ARG
    assert "share device" in N.last_error()
    assert lib.fl_init(2, (C.c_int32 * 2)(1, -1)) == N.FL_ERR_ARG
    import torch
    if torch.cuda.device_count() == 0:
        assert lib.fl_init(2, None) == N.FL_ERR_CUDA
    from conftest import model_image
    from dotnetfoundryllm_b200 import gguf
    d = loader.build_desc(gguf.parse(model_image("tiny")), tp_rank=N.FL_TP_ALL, tp_size=1)
    h = C.c_void_p()
    assert lib.fl_model_create(C.byref(d), C.byref(h)) == N.FL_ERR_UNSUPPORTED
    assert "group" in N.last_error()
