"""Tensor parallelism without a GPU: the weight shards a rank keeps (rows or
whole-block columns of the raw GGUF bytes) decode to exactly the matching
slice of the full tensor, the model descriptor is validated before any
device work, and the host-side handle exchange delivers every rank's handle
in rank order (gloo, world size 2)."""
from __future__ import annotations

import ctypes as C
import os
import socket

import numpy as np
import pytest

from dotnetfoundryllm_b200 import _native as N
from dotnetfoundryllm_b200 import ggufgen, runtime
from oracle import oracle as O

T_Q8_0, T_Q4_K, T_Q5_K, T_Q6_K = 8, 12, 13, 14


def _slice(t, raw, rows, cols, dim, rank, T):
    be = 32 if t == T_Q8_0 else 256
    bb = {T_Q8_0: 34, T_Q4_K: 144, T_Q5_K: 176, T_Q6_K: 210}[t]
    n = (rows // T) * cols if dim == 0 else rows * (cols // T)
    out = np.zeros(n // be * bb, dtype=np.uint8)
    runtime.check(N.cuda().fl_tp_slice(t, rows, cols, dim, rank, T, raw.ctypes.data_as(C.c_void_p),
                                       out.ctypes.data_as(C.c_void_p)), "fl_tp_slice")
    return out


def _deq(t, raw, n):
    rc, out = O.dequantize(t, raw, n)
    assert rc == 0
    return out


@pytest.mark.parametrize("t", [T_Q4_K, T_Q5_K, T_Q6_K, T_Q8_0])
@pytest.mark.parametrize("T", [2, 4])
def test_shards_decode_to_the_full_tensors_slices(t, T):
    rows, cols = 64, 2048
    raw = ggufgen.random_blocks(t, rows * cols, 5, t)
    full = _deq(t, raw, rows * cols).reshape(rows, cols)
    for rank in range(T):
        r = _slice(t, raw, rows, cols, 0, rank, T)
        np.testing.assert_array_equal(_deq(t, r, rows // T * cols).reshape(rows // T, cols),
                                      full[rank * rows // T:(rank + 1) * rows // T])
        c = _slice(t, raw, rows, cols, 1, rank, T)
        np.testing.assert_array_equal(_deq(t, c, rows * cols // T).reshape(rows, cols // T),
                                      full[:, rank * cols // T:(rank + 1) * cols // T])


def test_columns_must_split_into_whole_blocks():
    raw = ggufgen.random_blocks(T_Q4_K, 16 * 512, 1, 1)
    out = np.zeros(raw.size, dtype=np.uint8)
    rc = N.cuda().fl_tp_slice(T_Q4_K, 16, 512, 1, 0, 4, raw.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p))
    assert rc == N.FL_ERR_ARG


def _desc(**kw):
    from dotnetfoundryllm_b200 import gguf, loader
    d = loader.build_desc(gguf.parse(ggufgen.build_model(ggufgen.SPECS["tiny"])))
    for k, v in kw.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw,code", [
    (dict(tp_size=3), N.FL_ERR_UNSUPPORTED),
    (dict(tp_size=16), N.FL_ERR_UNSUPPORTED),
    (dict(tp_size=2, tp_rank=2), N.FL_ERR_ARG),
    (dict(tp_size=4), N.FL_ERR_UNSUPPORTED),  # tiny has 2 kv heads
])
def test_descriptor_validation(kw, code):
    h = C.c_void_p()
    assert N.cuda().fl_model_create(C.byref(_desc(**kw)), C.byref(h)) == code


class _FakeSession:
    def __init__(self, rank):
        self.rank = rank
        self.connected = None

    def tp_handle(self):
        return bytes([self.rank + 1]) * N.FL_TP_HANDLE_BYTES

    def tp_connect(self, handles):
        self.connected = handles


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)

    def gather(b):
        out = [None] * world
        dist.all_gather_object(out, b)
        return out

    s = _FakeSession(rank)
    runtime.connect_tensor_parallel(s, gather)
    q.put((rank, s.connected))
    dist.destroy_process_group()


def test_handle_exchange_in_rank_order_gloo():
    import torch.multiprocessing as mp
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get() for _ in procs)
    for p in procs:
        p.join(60)
    expect = [bytes([1]) * N.FL_TP_HANDLE_BYTES, bytes([2]) * N.FL_TP_HANDLE_BYTES]
    assert got[0] == expect and got[1] == expect
