"""Tensor parallelism on 2, 4 and 8 GPUs (as many as the box has) against
the CPU restatement.

Each family's GGUF is run by the oracle (single process, the reference's
algorithm) and by 2-8 ranks of the token kernel, each holding its shard and
exchanging partial sums and the argmax over NVLink.  Same bars as the
single-GPU parity tests: logits within 1e-3 + 1e-2·|ref| at every
teacher-forced step, greedy tokens identical, the device loop equal to the
host loop; every rank must see identical (full-vocabulary) logits; and the
same after the prompt went through the tensor-parallel prompt path.
"""
from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from dotnetfoundryllm_b200 import ggufgen
from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 1e-3
N_PROMPT, N_GEN = 48, 64
WORKER = Path(__file__).resolve().parent / "tp_worker.py"


def _gpus() -> int:
    import torch
    return torch.cuda.device_count()


@pytest.mark.parametrize("name,ranks", [("small-tp", 2), ("tiny-gemma2", 2), ("small-tp", 4), ("small-tp", 8)])
def test_ranks_match_the_oracle(name, ranks, tmp_path):
    if _gpus() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    img = ggufgen.build_model(ggufgen.SPECS[name])
    m = O.Model(img)
    prompt = ggufgen.prompt_ids(N_PROMPT, m.vocab, 1)
    toks, logs = m.generate_greedy(prompt, N_GEN, collect_logits=True)
    m.close()
    np.savez(tmp_path / "ref.npz", prompt=prompt, toks=np.array(toks))
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={ranks}",
           "--master-addr=127.0.0.1", f"--master-port={port}", str(WORKER), "--model", name,
           "--ref", str(tmp_path / "ref.npz"), "--out", str(tmp_path)]
    subprocess.run(cmd, env=env, timeout=900, check=True)
    rs = [np.load(tmp_path / f"rank{r}.npz") for r in range(ranks)]
    r0, r1 = rs[0], rs[-1]
    for r in rs[1:]:
        np.testing.assert_array_equal(r["logits"], r0["logits"])
    got = r0["logits"]
    err = np.abs(got - logs)
    bound = ATOL + RTOL * np.abs(logs)
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), f"{name}: step {worst[0]} id {worst[1]}: {got[worst]} vs {logs[worst]}"
    assert (r0["argmax"] == np.argmax(got, axis=1)).all()
    n = min(len(r0["greedy"]), len(toks))
    diverge = next((i for i in range(n) if r0["greedy"][i] != toks[i]), None)
    assert diverge is None or diverge >= 32, f"{name}: greedy token {diverge} differs"
    np.testing.assert_array_equal(r0["device"], r0["greedy"][:32])
    np.testing.assert_array_equal(r1["device"], r0["device"])
    # after the tensor-parallel prompt path
    np.testing.assert_array_equal(r0["pf_logits"], r1["pf_logits"])
    err = np.abs(r0["pf_logits"] - logs)
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), f"{name} prefill: step {worst[0]} id {worst[1]}: {r0['pf_logits'][worst]} vs {logs[worst]}"


def test_a_rank_that_misses_a_step_times_out_fast_and_the_group_recovers(tmp_path):
    """Failure detection without a GPU fault: rank 1 skips one step, so rank
    0's token kernel never sees rank 1's row words of the step's first
    exchange.  That bounded wait gives up after ~2 s and every later exchange
    of the step returns at once, so the call fails with FL_ERR_TIMEOUT in a
    few seconds (not one limit per exchange: 2 per layer + the argmax).  After
    fl_session_tp_reset on both ranks (which also clears the receive words,
    whose tags restart) the teacher-forced logits match the oracle again,
    identical on both ranks."""
    ranks = 2
    if _gpus() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    name = "small-tp"
    img = ggufgen.build_model(ggufgen.SPECS[name])
    m = O.Model(img)
    prompt = ggufgen.prompt_ids(16, m.vocab, 6)
    toks, logs = m.generate_greedy(prompt, 8, collect_logits=True)
    m.close()
    np.savez(tmp_path / "ref.npz", prompt=prompt, toks=np.array(toks))
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={ranks}",
           "--master-addr=127.0.0.1", f"--master-port={port}", str(WORKER), "--model", name,
           "--ref", str(tmp_path / "ref.npz"), "--out", str(tmp_path), "--scenario", "lost-step"]
    subprocess.run(cmd, env=env, timeout=600, check=True)
    r0, r1 = (np.load(tmp_path / f"rank{r}.npz") for r in range(ranks))
    assert bool(r0["timed_out"]), "the step without its peer did not report FL_ERR_TIMEOUT"
    assert float(r0["elapsed"]) < 10.0, f"timed-out step took {float(r0['elapsed']):.1f} s"
    np.testing.assert_array_equal(r0["logits"], r1["logits"])
    err = np.abs(r0["logits"] - logs)
    assert (err <= ATOL + RTOL * np.abs(logs)).all()


def test_two_ranks_in_one_process(tmp_path):
    """A host that keeps every rank in one process (the C# engine), one thread
    per GPU: the exchange regions are mapped with peer access instead of CUDA
    IPC.  Teacher-forced logits against the oracle, identical on both ranks."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    import threading

    from dotnetfoundryllm_b200 import loader, runtime
    name = "small-tp"
    img = ggufgen.build_model(ggufgen.SPECS[name])
    m = O.Model(img)
    prompt = ggufgen.prompt_ids(24, m.vocab, 2)
    toks, logs = m.generate_greedy(prompt, 16, collect_logits=True)
    m.close()
    models = [loader.load(img, device=r, tp_rank=r, tp_size=2) for r in range(2)]
    fwds = [runtime.CudaForwardPass(mo) for mo in models]
    handles = [f.tp_handle() for f in fwds]
    for f in fwds:
        f.tp_connect(handles)
    feed = [int(t) for t in prompt] + [int(t) for t in toks[:-1]]
    got = [[], []]
    errors = []
    gate = threading.Barrier(2)

    def run(r):
        try:
            kv = object()
            for pos, tok in enumerate(feed):
                gate.wait()
                want = pos >= len(prompt) - 1
                fwds[r].forward(tok, pos, kv, want_logits=want)
                if want:
                    got[r].append(fwds[r].logits.copy())
        except Exception as e:  # noqa: BLE001
            errors.append(e)
            gate.abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=600)
    try:
        assert not errors, errors
        a, b = np.stack(got[0]), np.stack(got[1])
        np.testing.assert_array_equal(a, b)
        err = np.abs(a - logs)
        assert (err <= ATOL + RTOL * np.abs(logs)).all()
    finally:
        for f in fwds:
            f.close()
        for mo in models:
            mo.close()


def test_two_ranks_on_one_device_are_refused():
    """Ranks wait on one another inside their kernels, so two on one GPU are
    refused at connect time, before any kernel runs."""
    if _gpus() < 1:
        pytest.skip("needs a GPU")
    from dotnetfoundryllm_b200 import loader, runtime
    img = ggufgen.build_model(ggufgen.SPECS["small-tp"])
    models = [loader.load(img, device=0, tp_rank=r, tp_size=2) for r in range(2)]
    fwds = [runtime.CudaForwardPass(mo) for mo in models]
    try:
        handles = [f.tp_handle() for f in fwds]
        with pytest.raises(runtime.ArgumentError, match="share device"):
            fwds[0].tp_connect(handles)
    finally:
        for f in fwds:
            f.close()
        for mo in models:
            mo.close()


def test_group_driven_from_one_thread():
    """fl_init + a model loaded with tp_rank FL_TP_ALL: the shim creates and
    connects one rank per GPU and runs each call on all of them, so a single
    host thread (the reference's Forward loop) drives tensor parallelism.
    Prompt path, token loop and device greedy loop against the oracle; a bad
    call is refused before any rank launches and the group keeps working."""
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    from dotnetfoundryllm_b200 import _native as N
    from dotnetfoundryllm_b200 import loader, runtime
    img = ggufgen.build_model(ggufgen.SPECS["small-tp"])
    m = O.Model(img)
    prompt = ggufgen.prompt_ids(24, m.vocab, 4)
    n_gen = 16
    toks, logs = m.generate_greedy(prompt, n_gen, collect_logits=True)
    m.close()
    runtime.init_tensor_parallel(2, [0, 1])
    model = loader.load(img, tp_rank=N.FL_TP_ALL, tp_size=2)
    fwd = runtime.CudaForwardPass(model)
    try:
        p = len(prompt) - 1
        feed = [int(prompt[-1])] + [int(t) for t in toks[:-1]]
        bound = ATOL + RTOL * np.abs(logs)
        for path in ("prompt path", "token loop"):
            kv = object()
            if path == "prompt path":
                fwd.prefill(prompt[:-1], 0, kv)
            else:
                for i in range(p):
                    fwd.forward(int(prompt[i]), i, kv, want_logits=False)
            got = []
            for s, tok in enumerate(feed):
                am = fwd.forward(tok, p + s, kv)
                got.append(fwd.logits.copy())
                assert am == int(np.argmax(got[-1]))
            err = np.abs(np.stack(got) - logs)
            worst = np.unravel_index(np.argmax(err - bound), err.shape)
            assert (err <= bound).all(), f"{path}: step {worst[0]} id {worst[1]}"
        # the device-resident greedy loop after the prompt path
        kv = object()
        fwd.prefill(prompt[:-1], 0, kv)
        dev = fwd.decode_greedy(int(prompt[-1]), p, n_gen)
        d = next((i for i in range(n_gen) if int(dev[i]) != int(toks[i])), None)
        if d is not None:
            srt = np.sort(logs[d])
            assert srt[-1] - srt[-2] < 1e-3, f"greedy token {d} differs"
        with pytest.raises(runtime.ArgumentOutOfRangeError):
            fwd.forward(model.desc.vocab, p + n_gen, kv)
        with pytest.raises(runtime.ArgumentError):
            fwd.forward(1, p + n_gen + 5, kv)
        with pytest.raises(runtime.NotSupportedError):
            fwd.profile_step(1, p + n_gen)
        fwd.forward(int(dev[-1]), p + n_gen, kv)
        assert np.isfinite(fwd.logits).all()
        ids, vals, _ = fwd.topk(5)
        assert int(ids[0]) == int(np.argmax(fwd.logits))
    finally:
        fwd.close()
        model.close()
