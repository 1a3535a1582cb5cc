"""Throughput of the GPT training step (forward, backward, clip_grad_norm_, AdamW) on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N

Workload: the GPT-2-small-shape configuration (12 layers, d_model 768, 12 heads, block 1024,
vocab 50304, tied head), micro-batch 8 sequences of 1024 tokens per GPU, AdamW (lr 3e-4,
wd 1e-4) with gradient clipping at 1.0, fp32 parameters; token ids uniform from a seed
(synthetic, no dataset). Data parallel over N GPUs (one process per GPU, NCCL all-reduce of
the gradient buffer), weak scaling: each GPU processes its own 8 x 1024 tokens.

Prints one JSON line (rank 0). ``value`` is tokens/s of the whole job with the token ids
already in device memory; ``e2e`` is the same step through the public API from pinned host
arrays (uploads and the loss read-back inside the timed region). ``roofline`` is the
tensor-core GEMM (the dominant kernel), timed live with CUDA events around every launch in
the timed region. ``cpu_baseline`` is the float32 NumPy restatement of the reference's step
(the oracle) on a bounded sample, timed on this host's cores.

``--impl reference`` times that CPU implementation alone (rank 0; other ranks exit 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

GPT2 = dict(vocab_size=50304, block_size=1024, n_layer=12, n_head=12, n_embd=768)
MICRO_BATCH = 8
SEQ = 1024
METRIC = "GPT fwd+bwd+AdamW tokens/s"
WORKLOAD = ("GPT-2-small-shape train step: 12 layers, d_model 768, 12 heads, block 1024, "
            "vocab 50304, tied head; micro-batch 8 x 1024 tokens per GPU; AdamW lr 3e-4 wd 1e-4, "
            "clip 1.0")


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    return p.parse_args()


def peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f) | {"source": "measured"}
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback"}


# ----------------------------------------------------------------------------- CPU leg
def cpu_reference_step_fn(threads: int):
    """A callable running one oracle step (float32 NumPy, the reference's algorithm) on one
    1024-token sequence of the workload, and a description of that sample."""
    import numpy as np
    from threadpoolctl import threadpool_limits

    from oracle import gpt as ogpt

    cfg = ogpt.Config(**GPT2)
    params = {k: v.astype(np.float32) for k, v in ogpt.init_params(cfg, 1234).items()}
    state = {"params": params, "state": None}
    ids, targets = ogpt.synthetic_batch(cfg, 1, SEQ, 99)
    limiter = threadpool_limits(threads)

    def step() -> None:
        out = ogpt.train_step(state["params"], ids, targets, cfg, state["state"])
        state["params"], state["state"] = out["params"], out["state"]

    sample = (f"1 sequence x {SEQ} tokens of the workload (full 12-layer GPT-2-small model, "
              f"float32 NumPy restatement of the reference step), {threads} BLAS threads")
    return step, sample, limiter


def time_cpu(step, steps: int, budget_s: float) -> tuple[float, int]:
    """Median seconds per step over up to ``steps`` timed steps within ``budget_s``."""
    times: list[float] = []
    t_start = time.perf_counter()
    while len(times) < steps:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start + times[-1] > budget_s:
            break
    return statistics.median(times), len(times)


def cpu_baseline(budget_s: float = 30.0) -> dict:
    threads = os.cpu_count() or 1
    step, sample, _lim = cpu_reference_step_fn(threads)
    step()  # allocator and BLAS warm-up
    sec, n = time_cpu(step, 3, budget_s)
    return {"value": SEQ / sec, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{sample}; median of {n} steps after 1 warm-up"}


def run_reference(args: argparse.Namespace) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    step, sample, _lim = cpu_reference_step_fn(threads)
    t_warm = time.perf_counter()
    for _ in range(max(min(args.warmup, 1), 0)):
        step()
    warm = time.perf_counter() - t_warm
    sec, n = time_cpu(step, args.steps, budget_s=max(150.0 - warm, 10.0))
    value = SEQ / sec
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": n, "warmup": min(args.warmup, 1),
        "ms_per_step": 1e3 * sec, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": SEQ,
                   "parallelism": "host cores", "sample": sample},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{sample}; median of {n} steps"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(gpu_index)], stdout=self.file,
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.file.seek(0)
        rows = [r.split(", ") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9 for i in range(4)
                          if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(sm)}


# ----------------------------------------------------------------------------- our arm
def run_ours(args: argparse.Namespace) -> None:
    import numpy as np
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    import tensorgrad_b200 as tg
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import lib
    from tensorgrad_b200.distributed import GradientAllReduce, barrier, max_over_ranks

    tg.set_device(local)
    tg.manual_seed(1234)
    model = tg.nn.GPT(tg.nn.GPTConfig(**GPT2, dropout=0.0))
    params = list(model.parameters())
    opt = tg.optim.AdamW(params, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
    reducer = GradientAllReduce(params) if world > 1 else None

    rng = np.random.default_rng(1000 + rank)
    ids_np = rng.integers(0, GPT2["vocab_size"], size=(MICRO_BATCH, SEQ), dtype=np.int64)
    tgt_np = rng.integers(0, GPT2["vocab_size"], size=(MICRO_BATCH, SEQ), dtype=np.int64)
    ids_dev, tgt_dev = tg.Tensor(ids_np), tg.Tensor(tgt_np)
    ids_pin = device.pinned_empty(ids_np.shape, np.int64)
    tgt_pin = device.pinned_empty(tgt_np.shape, np.int64)
    ids_pin[...] = ids_np
    tgt_pin[...] = tgt_np

    def step(ids, targets):
        loss = tg.cross_entropy(model(ids), targets)
        opt.zero_grad()
        loss.backward()
        if reducer is not None:
            reducer.reduce()
        tg.optim.clip_grad_norm_(params, 1.0)
        opt.step()
        return loss

    def timed(k: int, fn) -> float:
        barrier()
        tg.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(k):
            fn()
        stop.record()
        stop.synchronize()
        barrier()
        return max_over_ranks(start.elapsed_time(stop) / 1e3)

    # Device-resident inputs: the value line.
    for _ in range(args.warmup):
        step(ids_dev, tgt_dev)
    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    gpu_index = int(phys[local]) if len(phys) > local and phys[local].strip().isdigit() else local
    clocks = ClockSampler(gpu_index)
    launches0 = int(lib.tg_launch_count())
    lib.tg_gemm_profile(1)
    sec = timed(args.steps, lambda: step(ids_dev, tgt_dev))
    lib.tg_gemm_profile(0)
    launches = int(lib.tg_launch_count()) - launches0
    clock = clocks.stop()
    import ctypes

    gms, gl, gfl = ctypes.c_double(), ctypes.c_int64(), ctypes.c_double()
    lib.tg_gemm_profile_read(ctypes.byref(gms), ctypes.byref(gl), ctypes.byref(gfl))

    # End to end: pinned host ids/targets uploaded inside the step, loss read back.
    losses = []

    def e2e_step():
        losses.append(step(ids_pin, tgt_pin).item())

    for _ in range(args.warmup):
        e2e_step()
    sec_e2e = timed(args.steps, e2e_step)

    tokens = MICRO_BATCH * SEQ * world
    pk = peaks()
    achieved = gfl.value / (gms.value / 1e3) / 1e12 if gms.value > 0 else 0.0
    peak = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")))
    out = {
        "metric": METRIC,
        "value": tokens * args.steps / sec,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * sec / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic token ids (uniform, seeded); GPT-2 init from the seeded host RNG",
        "config": {"workload": WORKLOAD, "global_batch": MICRO_BATCH * world, "seq_len": SEQ,
                   "parallelism": f"dp{world}",
                   "matmul": "tcgen05 kind::tf32 with a 3xTF32 split (fp32-level accuracy)",
                   "l2": "no flush: every step streams several GB of activations, >> 126 MB L2"},
        "roofline": {
            "kernel": "tensor-core GEMM (gemm_tc_kernel, 3xTF32)",
            "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak if peak else None, "traffic": None,
            "peak_source": f"{pk['source']} bf16_tflops_sustained (dense bf16 cuBLAS)",
            "launches": gl.value, "device_ms_per_step": gms.value / args.steps,
            "tf32_ceiling_frac": achieved / (peak / 2) if peak else None,
            "tf32x3_ceiling_frac": achieved / (peak / 6) if peak else None,
        },
        "clocks": clock,
        "e2e": {"value": tokens * args.steps / sec_e2e, "unit": "tokens/s",
                "h2d_bytes_per_step": int(ids_np.nbytes + tgt_np.nbytes),
                "d2h_bytes_per_step": 4 + 8},
        "gpu_launches": launches,
        "final_loss": losses[-1] if losses else None,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline()
    if reducer is not None:
        reducer.close()
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def main() -> None:
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
