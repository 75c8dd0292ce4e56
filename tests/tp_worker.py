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


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", required=True)
    ap.add_argument("--ref", required=True, help="npz with the prompt and the reference's greedy tokens")
    ap.add_argument("--out", required=True, help="output directory (rank<r>.npz)")
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
