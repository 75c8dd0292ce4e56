"""Decode benchmark: Llama-3-8B-architecture Q4_K_M-style GGUF, batch 1, greedy,
after a 2048-token prompt.

A step is one decode token through the device token loop (every layer's
fused dequant-matvecs, attention over the HBM KV cache, LM head and argmax).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

- ``value``: whole-job decode tok/s with the token loop resident on the device
  (K greedy steps as back-to-back CUDA-graph launches, CUDA events, max over
  ranks).  Weights (4.9 GB) are far larger than L2 (126 MB), so every step
  streams them from HBM.
- ``e2e``: the same metric through the public C ABI call ``fl_forward`` with
  the token id copied host→device and the argmax copied back every step.
- ``roofline``: the step's one kernel, fl_token_kernel (persistent, one launch
  per token): algorithmic bytes per launch (GGUF weight bytes + the K/V rows
  read) ÷ its CUDA-event launch duration, against the measured HBM copy
  bandwidth in MEASURED_PEAKS.json; ``matvec_phase_gbs`` is the weight stream
  rate of its matvec phases alone (device timestamps at phase boundaries).
- ``cpu_baseline``: the C restatement of the reference CPU path (oracle/),
  all host threads, on a bounded sample: 2 of the 32 decoder layers at the same
  position plus the LM head, extrapolated to the full model.
- ``prefill``: the 2047 prompt tokens before the last through fl_prefill (one
  GPU or replicas; max of 3 device-timed passes after 2 warm-up passes, and
  one through the public call), against the measured dense bf16 tensor peak.
- ``--impl reference``: that CPU path alone, timed per step the same way.

With N > 1 GPUs (torchrun, one rank per GPU) the model is tensor-parallel by
default: every rank holds 1/N of the weights and the ranks exchange partial
sums and the argmax over NVLink inside the token kernel, so one decode stream
runs N times wider (strong scaling).  ``--parallel replicas`` runs N
independent replicas instead (weak scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIG = "llama3-8b"
PROMPT = 2048
# --model: the decode line's model (BASELINE configs[1] by default); name, quantization, weights per step
MODELS = {
    "llama3-8b": ("Llama-3-8B-arch Q4_K_M-style GGUF", "Q4_K/Q6_K", "4.9 GB"),
    "gemma2-9b": ("Gemma-2-9B-arch Q5_K/Q6_K GGUF", "Q5_K/Q6_K", "6.5 GB"),
    "mistral-7b": ("Mistral-7B-arch Q8_0 GGUF", "Q8_0", "7.6 GB"),
}
METRIC = "decode tok/s, Llama-3-8B-arch Q4_K_M-style GGUF, bs=1 greedy after a 2048-token prompt"
NOMINAL_HBM_GBS = 8000.0
PREFILL_WARMUP, PREFILL_TIMED = 2, 3


def set_model(name: str, prompt: int) -> None:
    """The decode line's model and metric string (the default keeps the headline's)."""
    global CONFIG, METRIC
    CONFIG = name
    METRIC = f"decode tok/s, {MODELS[name][0]}, bs=1 greedy after a {prompt}-token prompt"


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = tempfile.NamedTemporaryFile(prefix="clocks_", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu)], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.close()
        rows = []
        for line in Path(self.out.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.out.name)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": reasons}


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch
        import torch.distributed as dist
        # NCCL's log (with NCCL_DEBUG set, rank 0 prints its version line on
        # stdout) goes to a file, so stdout carries only the result line
        os.environ.setdefault("NCCL_DEBUG_FILE", os.path.join(tempfile.gettempdir(), "bench_nccl.%h.%p.log"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def gather_bytes(b: bytes, ws: int) -> list[bytes]:
    """Every rank's bytes in rank order (host-side channel for the TP handles)."""
    import torch.distributed as dist
    global _GLOO
    if "_GLOO" not in globals():
        _GLOO = dist.new_group(backend="gloo")
    out = [None] * ws
    dist.all_gather_object(out, b, group=_GLOO)
    return out


def allreduce_max(v: float, ws: int) -> float:
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws: int):
    """Host-synchronizing barrier (gloo): every rank's host thread leaves it
    together, so no rank's first timed kernel waits on a late peer."""
    if ws > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        global _GLOO
        if "_GLOO" not in globals():
            _GLOO = dist.new_group(backend="gloo")
        dist.barrier(group=_GLOO)


def spec(args):
    """The benchmark model; --layers keeps every matrix shape but fewer blocks
    (used only to size profiler captures)."""
    import dataclasses

    from dotnetfoundryllm_b200 import ggufgen
    s = ggufgen.SPECS[CONFIG]
    if args.layers:
        s = dataclasses.replace(s, n_layers=args.layers)
    return s


def model_image(args, ws: int, rank: int) -> np.ndarray:
    from dotnetfoundryllm_b200 import ggufgen
    if ws == 1:
        return ggufgen.build_model(spec(args))
    path = Path(tempfile.gettempdir()) / f"foundry_bench_{CONFIG}_{os.environ.get('MASTER_PORT', '0')}.gguf"
    if rank == 0:
        ggufgen.build_model(spec(args), str(path))
    barrier(ws)
    img = np.fromfile(path, dtype=np.uint8)
    barrier(ws)
    if rank == 0:
        path.unlink(missing_ok=True)
    return img


def cpu_sample(img: np.ndarray, position: int, repeats: int = 3, threads: int | None = None) -> dict:
    """Oracle timing on 2 decoder layers + the LM head; per-token estimate."""
    from oracle import oracle as O
    threads = threads or os.cpu_count() or 1
    O.set_threads(threads)
    m = O.Model(img, max_layers=2)
    s = O.Session(m)
    s.fake_length(position)
    t_layers, t_head = [], []
    for _ in range(repeats):
        s.fake_length(position)
        t0 = time.perf_counter()
        rc = s.forward_layers(1, position, 2)
        t1 = time.perf_counter()
        rc2 = s.forward_head()
        t2 = time.perf_counter()
        assert rc == 0 and rc2 == 0, (rc, rc2)
        t_layers.append(t1 - t0)
        t_head.append(t2 - t1)
    n_layers = m.n_layers
    per_tok = (min(t_layers) / 2) * n_layers + min(t_head)
    # the reference's own loop has no parallelism: the same sample on one thread
    O.set_threads(1)
    s.fake_length(position)
    t0 = time.perf_counter()
    rc = s.forward_layers(1, position, 2)
    t1 = time.perf_counter()
    rc2 = s.forward_head()
    t2 = time.perf_counter()
    assert rc == 0 and rc2 == 0, (rc, rc2)
    O.set_threads(threads)
    per_tok_1 = (t1 - t0) / 2 * n_layers + (t2 - t1)
    s.close()
    m.close()
    return {"tok_s": 1.0 / per_tok, "per_token_s": per_tok, "threads": threads, "layer_s": min(t_layers) / 2,
            "head_s": min(t_head), "n_layers": n_layers, "tok_s_1thread": 1.0 / per_tok_1}


def decode_workload(pos_timed: int, steps: int, prompt: int) -> str:
    """config.workload of the decode line, the same string on both arms."""
    return (f"{CONFIG} {MODELS[CONFIG][1]} bs=1 greedy decode, positions {pos_timed}..{pos_timed + steps - 1} "
            f"after a {prompt}-token prompt")


def decode_config(args, ws: int, pos_timed: int, streams: int = 1) -> dict:
    """The decode line's config, the same dict on both arms for the same launch."""
    tp = ws > 1 and args.parallel == "tp"
    return {"workload": decode_workload(pos_timed, args.steps, args.prompt),
            "model": CONFIG, "global_batch": streams, "seq_len": args.prompt,
            "parallelism": f"tp{ws}" if tp else (f"replicas x{ws}" if ws > 1 else "single GPU"),
            "l2": f"inputs larger than L2 ({MODELS[CONFIG][2]} of weights per step)"}


def run_reference(args, ws, rank):
    if rank != 0:
        return
    from dotnetfoundryllm_b200 import ggufgen
    img = ggufgen.build_model(spec(args))
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    m = O.Model(img, max_layers=2)
    s = O.Session(m)
    pos = args.prompt - 1
    times = []
    for i in range(args.warmup + args.steps):
        s.fake_length(pos + i)
        t0 = time.perf_counter()
        s.forward_layers(1, pos + i, 2)
        t1 = time.perf_counter()
        s.forward_head()
        t2 = time.perf_counter()
        if i >= args.warmup:
            times.append((t1 - t0) / 2 * m.n_layers + (t2 - t1))
    # the reference's own Forward loop is single-threaded (LlamaForwardPass.cs:29): one step on one thread
    O.set_threads(1)
    s.fake_length(pos + args.warmup)
    t0 = time.perf_counter()
    s.forward_layers(1, pos + args.warmup, 2)
    t1 = time.perf_counter()
    s.forward_head()
    t2 = time.perf_counter()
    one_thread = 1.0 / ((t1 - t0) / 2 * m.n_layers + (t2 - t1))
    s.close()
    m.close()
    per = sum(times) / len(times)
    value = 1.0 / per
    pos_timed = pos + args.warmup
    sample = (f"C restatement of the reference CPU path on all {threads} host threads (the reference itself is "
              f"single-threaded: single_thread_value); per step 2 of {m.n_layers} decoder layers (F32 weights "
              f"dequantized at load, as the reference does) at positions {pos_timed}.."
              f"{pos_timed + args.steps - 1} plus the LM head, layer time x{m.n_layers // 2}")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init GGUF)",
        "config": decode_config(args, ws, pos_timed, 1 if (ws == 1 or args.parallel == "tp") else ws),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample,
                         "single_thread_value": one_thread},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def prefill_flops(d, n: int) -> float:
    """Algorithmic FLOPs of a prompt of n tokens from position 0: the
    projections of every layer but the last (whose outputs feed nothing), the
    last layer's q/k/v projection, and causal attention (q.k and p.v over
    n(n+1)/2 query-key pairs per head) in every layer but the last."""
    qd, kvd = d.n_heads * d.head_dim, d.n_kv_heads * d.head_dim
    h, f = d.hidden, d.ffn
    qkv = h * (qd + 2 * kvd)
    rest = qd * h + 3 * h * f
    mm = 2.0 * n * (d.n_layers * qkv + (d.n_layers - 1) * rest)
    attn = 4.0 * d.n_heads * d.head_dim * (n * (n + 1) / 2) * (d.n_layers - 1)
    return mm + attn


def prefill_record(p: dict, d, peaks: dict, ws: int, cpu: dict) -> dict:
    streams = p["streams"]  # prompts processed at once: 1 with tensor parallelism, N replicas otherwise
    fl = streams * prefill_flops(d, p["tokens"])
    tflops = fl / (p["ms"] / 1e3) / 1e12
    return {
        "path": "fl_prefill: split-fp16 GEMMs on the hand-written tcgen05 kernel (fl_tc_gemm) for the projections and for attention's "
                "QK^T and PV; own dequant, norm, RoPE/KV-append, masked-softmax and GLU kernels",
        "tokens": p["tokens"], "ms": p["ms"], "tok_s": streams * p["tokens"] / (p["ms"] / 1e3),
        "e2e_tok_s": streams * p["tokens"] / p["e2e_s"],
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": ws * peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tflops / (ws * peaks["bf16_tflops"]), "algorithmic_flops": fl,
                     "executed_tensor_flops_note": "the split-fp16 GEMMs run 3x the projection FLOPs",
                     "peak_source": peaks["source"]},
        "cpu_baseline": {"value": cpu["tok_s"], "unit": "tok/s", "cores": cpu["threads"], "kind": "port",
                         "sample": "the reference prefills with one Forward per prompt token: the decode "
                                   "cpu_baseline sample stands for its prompt rate"},
    }


def profiler_range(args):
    """With --profile-range: cudaProfilerStart now (the caller stops), through
    the CUDA runtime the native library uses; else None."""
    if not args.profile_range:
        return None
    import ctypes
    cudart = ctypes.CDLL("libcudart.so.12")
    cudart.cudaProfilerStart()
    return cudart


def run_batch(args):
    """Mistral-7B-architecture Q8_0, 32 concurrent
    sequences, each a 512-token random prompt (fl_prefill_seq into its own
    slot) followed by batched greedy decode steps (fl_forward_batch).  A step
    is one token of every sequence; timed on the host around synchronous
    calls (each copies the step's token ids in and the argmax out)."""
    from dotnetfoundryllm_b200 import ggufgen, loader, runtime
    B, P = 32, 512
    sp = ggufgen.SPECS["mistral-7b"]
    img = ggufgen.build_model(sp)
    max_ctx = P + args.warmup + args.steps + 8
    model = loader.load(img, device=0, max_ctx=max_ctx)
    fwd = runtime.CudaForwardPass(model, max_ctx=max_ctx, max_batch=B)
    d = model.desc
    prompts = [ggufgen.prompt_ids(P, d.vocab, 100 + b) for b in range(B)]
    t0 = time.perf_counter()
    for b in range(B):
        fwd.prefill_seq(b, prompts[b][:-1], 0)
    prefill_s = time.perf_counter() - t0
    pos = np.full(B, P - 1, np.int32)
    nxt = np.array([int(p[-1]) for p in prompts], np.int32)
    slots = np.arange(B, dtype=np.int32)
    for _ in range(args.warmup):
        nxt = fwd.forward_batch(nxt, pos, slots)
        pos += 1
    pos_timed = int(pos[0])
    cudart = profiler_range(args)
    clocks = ClockSampler(0)
    clocks.start()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        nxt = fwd.forward_batch(nxt, pos, slots)
        pos += 1
    dt = time.perf_counter() - t0
    clk = clocks.stop()
    if cudart:
        cudart.cudaProfilerStop()
    kvd = d.n_kv_heads * d.head_dim
    avg_ctx = pos_timed + args.steps / 2 + 1
    kv_bytes = B * d.n_layers * kvd * 4 * (2 * avg_ctx + 2)
    wbytes = model.weight_bytes()
    step_bytes = wbytes + kv_bytes
    ms = dt / args.steps * 1e3
    peaks = load_peaks()
    gbs = step_bytes / (ms / 1e3) / 1e9
    split_bytes = 4.0 * (wbytes / (34.0 / 32.0))  # Q8_0: 34 B per 32 weights; the [lo | hi] cache holds 4 B per weight
    print(json.dumps({
        "metric": "batched decode tok/s, Mistral-7B-arch Q8_0, 32 sequences, greedy after 512-token prompts",
        "value": B * args.steps / dt, "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init GGUF, N(0,0.02) weights)",
        "config": {"workload": f"mistral-7b Q8_0, {B} sequences, positions {pos_timed}..{pos_timed + args.steps - 1}",
                   "model": "mistral-7b", "global_batch": B, "seq_len": P, "parallelism": "single GPU"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "algorithmic_bytes_per_step": step_bytes,
                     "note": "algorithmic = Q8_0 weights + F32 K/V read and written; the step's GEMMs read the "
                             f"cached split-fp16 weights ({split_bytes / 1e9:.1f} GB per step)"},
        "prefill_s_32x511_tokens": prefill_s,
        "clocks": clk,
    }), flush=True)
    fwd.close()
    model.close()


def run_prefill_only(args):
    """The prompt path of the benchmark model alone (for profiler launch lists)."""
    from dotnetfoundryllm_b200 import ggufgen, loader, runtime
    img = ggufgen.build_model(spec(args))
    max_ctx = args.prompt + 64
    model = loader.load(img, device=0, max_ctx=max_ctx)
    fwd = runtime.CudaForwardPass(model, max_ctx=max_ctx)
    pre = ggufgen.prompt_ids(args.prompt, model.desc.vocab, 0)[:-1]
    kv = object()
    ms = [fwd.time_prefill(pre, 0, kv) for _ in range(args.warmup + args.steps)][args.warmup:]
    fl = prefill_flops(model.desc, len(pre))
    peaks = load_peaks()
    print(json.dumps({"metric": "prefill tok/s", "value": len(pre) / (max(ms) / 1e3), "unit": "tok/s",
                      "ms": max(ms), "tokens": len(pre), "tflops": fl / (max(ms) / 1e3) / 1e12,
                      "frac": fl / (max(ms) / 1e3) / 1e12 / peaks["bf16_tflops"]}), flush=True)
    fwd.close()
    model.close()


def run_ours(args, ws, rank, local):
    from dotnetfoundryllm_b200 import loader, runtime
    img = model_image(args, ws, rank)
    max_ctx = args.prompt + args.warmup + 2 * args.steps + 64
    tp = ws > 1 and args.parallel == "tp"
    model = loader.load(img, device=local, max_ctx=max_ctx, tp_rank=rank if tp else 0, tp_size=ws if tp else 1)
    fwd = runtime.CudaForwardPass(model, max_ctx=max_ctx)
    if tp:
        runtime.connect_tensor_parallel(fwd, lambda b: gather_bytes(b, ws))
    streams = 1 if tp else ws  # independent decode streams of the whole job
    from dotnetfoundryllm_b200 import ggufgen
    prompt = ggufgen.prompt_ids(args.prompt, model.desc.vocab, 0)
    kv = object()
    pre = prompt[:-1]
    # the prompt path (fl_prefill; tensor-parallel across the ranks with TP):
    # PREFILL_WARMUP + PREFILL_TIMED device-timed passes over the same 2047 tokens
    # (each starts from an empty KV cache), then one through the public call with
    # the token ids in host memory; the last one leaves the prompt's K/V in the
    # cache for the decode steps.  Max over ranks.
    barrier(ws)
    pf_ms = [fwd.time_prefill(pre, 0, kv) for _ in range(PREFILL_WARMUP + PREFILL_TIMED)][PREFILL_WARMUP:]
    barrier(ws)
    t0 = time.perf_counter()
    fwd.prefill(pre, 0, kv)
    pf_e2e_s = time.perf_counter() - t0
    prefill = {"ms": allreduce_max(max(pf_ms), ws), "e2e_s": allreduce_max(pf_e2e_s, ws), "tokens": len(pre),
               "streams": streams}
    pos = args.prompt - 1
    tok = int(prompt[-1])
    # warm-up (device-resident greedy loop)
    if args.warmup:
        out = fwd.decode_greedy(tok, pos, args.warmup)
        tok = int(out[-1])
        pos += args.warmup
    launches = fwd.launches_per_step()
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
    barrier(ws)
    cudart = profiler_range(args)
    ms = fwd.time_decode(tok, pos, args.steps)
    if cudart:
        cudart.cudaProfilerStop()
    clk = clocks.stop() if clocks else None
    ms_max = allreduce_max(ms, ws)
    pos_timed = pos
    pos += args.steps
    # e2e through the C ABI with host buffers
    barrier(ws)
    t0 = time.perf_counter()
    cur = tok
    for i in range(args.steps):
        cur = fwd.forward(cur, pos + i, kv, want_logits=False)
    e2e_s = time.perf_counter() - t0
    e2e_max = allreduce_max(e2e_s, ws)
    # the matvec phases alone (device timestamps at phase boundaries)
    profs = [fwd.profile_step(int(prompt[i % args.prompt]), pos + args.steps + i) for i in range(3)]
    mv_ms = min(p["ms"]["matvec"] for p in profs)
    mv_bytes = profs[0]["bytes"]["matvec"]
    peaks = load_peaks()
    mv_gbs = mv_bytes / (mv_ms / 1e3) / 1e9
    d = model.desc
    kvd = d.n_kv_heads * d.head_dim
    avg_ctx = pos_timed + args.steps / 2 + 1
    kv_bytes = d.n_layers * kvd * 4 * (2 * avg_ctx + 2)
    step_bytes = model.weight_bytes() + kv_bytes
    ms_per_step = ms_max / args.steps
    step_gbs = step_bytes / (ms_per_step / 1e3) / 1e9  # one launch per step
    value = streams * args.steps / (ms_max / 1e3)
    result = None
    if rank == 0:
        cpu = {"tok_s": None, "threads": 0} if args.no_cpu_baseline else cpu_sample(img, pos_timed)
        traffic, traffic_note = None, None
        tf = ROOT / "profiles" / "traffic.json"
        if tf.exists() and not args.layers and args.prompt == PROMPT:
            tj = json.loads(tf.read_text())
            if CONFIG in tj and not tp:
                # dram__bytes of one full launch of this workload, measured by ncu (profiles/)
                traffic = int(tj[CONFIG])
                traffic_note = (f"ncu dram__bytes_read + write of one full 32-layer launch at position "
                                f"{tj['position']} ({tj['ratio']:.4f} x its algorithmic bytes)")
            elif CONFIG in tj:
                # a rank streams its shard: the measured ratio applied to the rank's bytes
                traffic = int(step_bytes * tj["ratio"])
                traffic_note = "measured full-launch traffic/algorithmic ratio x this rank's bytes (per rank)"
        result = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if tp else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init GGUF, N(0,0.02) weights)",
            "config": decode_config(args, ws, pos_timed, streams),
            "roofline": {"bound": "hbm", "achieved": step_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": step_gbs / peaks["hbm_gbs"], "traffic": traffic,
                         "kernel": "fl_token_kernel (one persistent launch per token)",
                         "algorithmic_bytes_per_launch": step_bytes,
                         "peak_source": peaks["source"], "frac_of_nominal_8tbs": step_gbs / NOMINAL_HBM_GBS,
                         **({"traffic_note": traffic_note} if traffic_note else {}),
                         "matvec_phase_gbs": mv_gbs, "matvec_phase_frac": mv_gbs / peaks["hbm_gbs"]},
            "cpu_baseline": {"value": cpu["tok_s"], "unit": "tok/s", "cores": cpu["threads"], "kind": "port",
                             "sample": f"oracle (C restatement of the reference CPU path, F32 weights) on all "
                                       f"{cpu['threads']} host threads (the reference is single-threaded: "
                                       f"single_thread_value), 2 of 32 decoder layers at position {pos_timed} "
                                       "+ the LM head, layer time x16",
                             "single_thread_value": cpu.get("tok_s_1thread")},
            "e2e": {"value": streams * args.steps / e2e_max, "unit": "tok/s", "h2d_bytes_per_step": 16 * ws,
                    "d2h_bytes_per_step": 4 * ws},
            "gpu_launches": launches * args.steps,
            "clocks": clk,
            "prefill": prefill_record(prefill, d, peaks, ws, cpu),
        }
    barrier(ws)  # no rank frees its exchange region while a peer may still use it
    fwd.close()
    model.close()
    return result


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt length (default: the BASELINE 2048)")
    ap.add_argument("--layers", type=int, default=0, help="profiling only: fewer blocks, same matrix shapes")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="profiling only: skip the CPU sample")
    ap.add_argument("--workload", default="decode", choices=["decode", "batch"],
                    help="decode: the bs=1 headline (default); batch: Mistral-7B Q8_0, 32 sequences (BASELINE configs[2])")
    ap.add_argument("--profile-range", action="store_true",
                    help="profiling only: bracket the timed steps with cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="profiling only: the prompt path alone (one GPU), W + K device-timed passes")
    ap.add_argument("--parallel", default="tp", choices=["tp", "replicas"],
                    help="N > 1: tensor parallelism (default) or independent replicas")
    ap.add_argument("--model", default=CONFIG, choices=sorted(MODELS),
                    help="decode workload's model: llama3-8b (default, BASELINE configs[1]), gemma2-9b "
                         "(configs[3]: use --prompt 4096), mistral-7b")
    args = ap.parse_args()
    set_model(args.model, args.prompt)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), rank)
        return
    ws, rank, local = dist_setup()
    if args.prefill_only:
        run_prefill_only(args)
        return
    if args.workload == "batch":
        if rank == 0:
            run_batch(args)
        return
    res = run_ours(args, ws, rank, local)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
