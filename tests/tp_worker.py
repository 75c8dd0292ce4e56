"""One rank of the tensor-parallel parity run (launched by torchrun from
tests/test_gpu_tp.py): loads this rank's shard of a generated GGUF, connects
the ranks' sessions (handles gathered over a gloo group) and records, under
teacher forcing, the logits and argmax of every decode step, then the greedy
tokens of the host loop and of the device-resident loop, and the teacher-forced
logits again after the prompt went through the tensor-parallel fl_prefill."""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch.distributed as dist  # noqa: E402

from dotnetfoundryllm_b200 import ggufgen, loader, runtime  # noqa: E402


def _teacher_forced(fwd, prompt, toks):
    kv = object()
    for i in range(len(prompt) - 1):
        fwd.forward(int(prompt[i]), i, kv, want_logits=False)
    pos, out = len(prompt) - 1, []
    for tok in [int(prompt[-1])] + [int(t) for t in toks[:-1]]:
        fwd.forward(tok, pos, kv)
        out.append(fwd.logits.copy())
        pos += 1
    return np.stack(out)


def lost_step(fwd, prompt, toks, rank: int, out: str) -> None:
    """A rank that misses a step: the ranks run a few steps together, then
    every rank but 0 skips one.  Rank 0's step must fail with FL_ERR_TIMEOUT
    after about one wait limit (~2 s), not one per exchange of the step.
    After fl_session_tp_reset on every rank (between host barriers) the group
    runs the teacher-forced sequence again, as on a fresh session."""
    import time
    kv = object()
    for i in range(4):
        fwd.forward(int(prompt[i]), i, kv, want_logits=False)
    dist.barrier()
    elapsed, timed_out = 0.0, False
    if rank == 0:
        t0 = time.monotonic()
        try:
            fwd.forward(int(prompt[4]), 4, kv, want_logits=False)
        except runtime.DeviceTimeoutError:
            timed_out = True
        elapsed = time.monotonic() - t0
    dist.barrier()
    fwd.tp_reset()
    dist.barrier()
    logits = _teacher_forced(fwd, prompt, toks)
    np.savez(Path(out) / f"rank{rank}.npz", logits=logits, timed_out=np.array(timed_out),
             elapsed=np.array(elapsed))
    dist.barrier()
    fwd.close()
    dist.barrier()
    dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--ref", required=True, help="npz with the prompt and the reference's greedy tokens")
    ap.add_argument("--out", required=True, help="output directory (rank<r>.npz)")
    ap.add_argument("--scenario", default="parity", choices=["parity", "lost-step"])
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo")

    def gather(b: bytes) -> list[bytes]:
        out = [None] * world
        dist.all_gather_object(out, b)
        return out

    ref = np.load(args.ref)
    prompt, toks = ref["prompt"], ref["toks"]
    img = ggufgen.build_model(ggufgen.SPECS[args.model])
    model = loader.load(img, device=local, tp_rank=rank, tp_size=world)
    fwd = runtime.CudaForwardPass(model)
    runtime.connect_tensor_parallel(fwd, gather)
    if args.scenario == "lost-step":
        lost_step(fwd, prompt, toks, rank, args.out)
        return
    kv = object()
    for i in range(len(prompt) - 1):
        fwd.forward(int(prompt[i]), i, kv, want_logits=False)
    pos = len(prompt) - 1
    logits, argmax = [], []
    for tok in [int(prompt[-1])] + [int(t) for t in toks[:-1]]:
        argmax.append(fwd.forward(tok, pos, kv))
        logits.append(fwd.logits.copy())
        pos += 1
    greedy, _ = runtime.generate_greedy(fwd, prompt, len(toks))
    kv = object()
    for i in range(len(prompt) - 1):
        fwd.forward(int(prompt[i]), i, kv, want_logits=False)
    device = fwd.decode_greedy(int(prompt[-1]), len(prompt) - 1, 32)
    # the prompt path (tensor-parallel fl_prefill), then the same teacher-forced steps
    kv = object()
    fwd.prefill(prompt[:-1], 0, kv)
    pos = len(prompt) - 1
    pf_logits = []
    for tok in [int(prompt[-1])] + [int(t) for t in toks[:-1]]:
        fwd.forward(tok, pos, kv)
        pf_logits.append(fwd.logits.copy())
        pos += 1
    np.savez(Path(args.out) / f"rank{rank}.npz", logits=np.stack(logits), argmax=np.array(argmax),
             greedy=np.array(greedy), device=np.array(device), pf_logits=np.stack(pf_logits))
    dist.barrier()  # no rank unmaps or frees its exchange region while a peer may still use it
    fwd.close()
    model.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
