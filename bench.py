"""Throughput of the tensorgrad training step (forward, backward, AdamW) on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gpt2|char_gpt|mha|cnn|lstm|gru]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N

Workloads (synthetic seeded inputs of each configuration's shapes; no dataset):

* ``gpt2`` (default): GPT-2-small shape (12 layers, d_model 768, 12 heads, block 1024, vocab
  50304, tied head), micro-batch 8 x 1024 tokens per GPU, AdamW (lr 3e-4, wd 1e-4), clip 1.0.
  Data parallel over N GPUs (one process per GPU, NCCL all-reduce of the gradient arena),
  weak scaling.
* ``char_gpt``: 4 layers, d_model 128, 4 heads, block 128, vocab 65, batch 32; AdamW, clip 1.0.
* ``mha``: the fused causal attention op alone, forward + backward, Q/K/V/dO (16, 8, 512, 64).
* ``cnn``: Conv(3->32)-BN-ReLU-Pool, Conv(32->64)-BN-ReLU-Pool, Linear(16384->4) on 256
  images of 3x64x64; cross entropy; AdamW.
* ``lstm`` / ``gru``: the adding problem, T = 100, batch 512, hidden 512, Linear(512->1) on
  the last state, MSE; BPTT; AdamW.

Prints one JSON line (rank 0). ``value`` is the workload's throughput for the whole job with
the inputs already in device memory; ``e2e`` is the same step through the public API from
pinned host arrays (uploads and the read-back of the step's result inside the timed region).
``roofline`` is the tensor-core GEMM (the dominant kernel), timed live with CUDA events
around each of its launches in the timed region; its FLOPs are algorithmic (causal products
counted at half). ``cpu_baseline`` is the float32 NumPy restatement of the reference's step
(the oracle) on a bounded sample, timed on this host's cores.

``--impl reference`` times that CPU implementation alone (rank 0; other ranks exit 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from dataclasses import dataclass, field
from typing import Any

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ADAMW = dict(lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="gpt2")
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--no-hbm", action="store_true",
                   help="skip the per-kernel HBM roofline leg (HBM-bound kernels timed alone)")
    p.add_argument("--gemm", metavar="M,N,K,TA,TB",
                   help="time one fp32 tg_gemm of this shape instead of a training step "
                        "(a kernel probe: C = op(A) op(B), TA/TB = 1 for transposed storage)")
    p.add_argument("--matmul-precision", choices=["3xtf32", "tf32"], default="3xtf32",
                   help="tensor-core precision of the --gemm probe (tf32: one MMA per product, "
                        "the kernel's raw TF32 rate)")
    p.add_argument("--layers", type=int, default=None,
                   help="GPT workloads: fewer layers (a smaller case of the same kernels, for "
                        "profiler captures); the JSON line names the change")
    p.add_argument("--batch", type=int, default=None,
                   help="GPT workloads: a smaller micro-batch (profiler captures)")
    return p.parse_args()


def run_gemm(args: argparse.Namespace) -> None:
    """Time ``tg_gemm`` alone on one shape (device-resident N(0,1) operands, CUDA events)."""
    import numpy as np
    import torch

    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import check, lib

    m, n, k, ta, tb = (int(v) for v in args.gemm.split(","))
    rng = np.random.default_rng(0)
    a = device.from_numpy(rng.standard_normal((k, m) if ta else (m, k)).astype(np.float32))
    b = device.from_numpy(rng.standard_normal((n, k) if tb else (k, n)).astype(np.float32))
    c = device.empty((m, n), np.float32)

    def call() -> None:
        check(lib.tg_gemm(0, ta, tb, m, n, k, 1.0, a.ptr, m if ta else k, b.ptr,
                          k if tb else n, 0.0, c.ptr, n, None, device.stream()), "gemm")

    check(lib.tg_set_matmul_precision(1 if args.matmul_precision == "tf32" else 0))
    for _ in range(args.warmup):
        call()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        call()
    stop.record()
    stop.synchronize()
    ms = start.elapsed_time(stop) / max(args.steps, 1)
    print(json.dumps({"metric": f"fp32 GEMM TFLOP/s ({args.matmul_precision})",
                      "value": 2.0 * m * n * k / ms / 1e9,
                      "unit": "TFLOP/s", "ms_per_call": ms, "shape": [m, n, k, ta, tb],
                      "steps": args.steps, "warmup": args.warmup}), flush=True)


# roofline.traffic: bytes read + written in DRAM per tensor-core GEMM launch, averaged over
# the launches of one training step in an ncu capture (a capture cannot run inside the bench).
GEMM_TRAFFIC_PER_LAUNCH = {"gpt2": 163.8e6}


def peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f) | {"source": "measured"}
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback"}


# ----------------------------------------------------------------------------- workloads
@dataclass
class Built:
    """A workload instantiated on the device."""

    step: Any                     # step(inputs) -> result (a Tensor or tuple of them)
    dev_inputs: tuple             # inputs already in device memory
    pinned_inputs: tuple          # the same inputs in page-locked host memory
    h2d_bytes: int
    d2h_bytes: int                # bytes of the result read back per step (e2e)
    params: list = field(default_factory=list)


@dataclass
class Workload:
    name: str
    metric: str
    unit: str
    units_per_step: int           # tokens / samples / calls one GPU processes per step
    description: str
    config: dict

    def flops(self) -> float:
        return 0.0


def _train_step(tg, model_fn, params, loss_fn, reducer, clip: float | None):
    opt = tg.optim.AdamW(params, **ADAMW)

    def step(*inputs):
        loss = loss_fn(model_fn(inputs[0]), inputs[1])
        opt.zero_grad()
        loss.backward()
        if reducer is not None:
            reducer.reduce()
        if clip is not None:
            tg.optim.clip_grad_norm_(params, clip, sync=False)
        opt.step()
        return loss

    return step


class _AsyncReadback:
    """The end-to-end read of each step's result without a blocking wait: right after the
    step, one asynchronous device-to-host copy per result tensor into page-locked buffers
    (two sets, used in turn) with an event behind them. A set is reused only after its event
    (two steps back) has completed, and the values are taken once the timed region has been
    synchronised. With a blocking read the host could queue the next step only after the
    device had finished this one; here it queues it while the device works."""

    def __init__(self, lib, device) -> None:
        self.lib, self.device = lib, device
        self.buffers: list = [None, None]
        self.events: list = [None, None]
        self.turn = 0
        self.last = None

    def issue(self, result) -> None:
        import time

        tensors = list(result) if isinstance(result, (list, tuple)) else [result]
        i = self.turn % 2
        self.turn += 1
        if self.events[i] is not None:
            while not self.events[i].query():
                time.sleep(0)
        if self.buffers[i] is None:
            self.buffers[i] = [self.device.pinned_empty(t.shape, t.dtype) for t in tensors]
        for t, buf in zip(tensors, self.buffers[i], strict=True):
            data = t.data
            if data.nbytes:
                rc = self.lib.tg_memcpy_d2h(buf.ctypes.data, data.ptr, data.nbytes,
                                            self.device.stream())
                if rc:
                    raise RuntimeError(f"device-to-host copy failed ({rc})")
        if self.events[i] is None:
            self.events[i] = self.device._Event()
        self.events[i].record()
        self.last = i

    def value(self):
        """The last result's host values (a float for a one-element result); call after the
        stream has been synchronised."""
        if self.last is None:
            return None
        bufs = self.buffers[self.last]
        return float(bufs[0].reshape(-1)[0]) if len(bufs) == 1 and bufs[0].size == 1 else None


def _pinned(device, arrays):
    import numpy as np

    out = []
    for a in arrays:
        p = device.pinned_empty(a.shape, a.dtype if a.dtype != np.float64 else np.float32)
        p[...] = a
        out.append(p)
    return tuple(out)


class GPTWorkload(Workload):
    def __init__(self, name, cfg: dict, batch: int, seq: int, description: str) -> None:
        super().__init__(name, "GPT fwd+bwd+AdamW tokens/s", "tokens/s", batch * seq,
                         description, {"global_batch": batch, "seq_len": seq})
        self.cfg, self.batch, self.seq = cfg, batch, seq

    def flops(self) -> float:
        from oracle import gpt as ogpt

        return ogpt.step_flops(ogpt.Config(**self.cfg), self.batch, self.seq)

    def build(self, tg, device, rank, reducer_cls) -> Built:
        import numpy as np

        tg.manual_seed(1234)
        model = tg.nn.GPT(tg.nn.GPTConfig(**self.cfg, dropout=0.0))
        params = list(model.parameters())
        reducer = reducer_cls(params) if reducer_cls else None
        step = _train_step(tg, model, params, tg.cross_entropy, reducer, 1.0)
        rng = np.random.default_rng(1000 + rank)
        v = self.cfg["vocab_size"]
        ids = rng.integers(0, v, size=(self.batch, self.seq), dtype=np.int64)
        tgt = rng.integers(0, v, size=(self.batch, self.seq), dtype=np.int64)
        return Built(step, (tg.Tensor(ids), tg.Tensor(tgt)), _pinned(device, (ids, tgt)),
                     ids.nbytes + tgt.nbytes, 4, params)

    def cpu_step(self, threads: int):
        import numpy as np

        from oracle import gpt as ogpt

        cfg = ogpt.Config(**self.cfg)
        batch = 1 if self.seq >= 1024 else self.batch
        params = {k: v.astype(np.float32) for k, v in ogpt.init_params(cfg, 1234).items()}
        state = {"params": params, "state": None}
        ids, targets = ogpt.synthetic_batch(cfg, batch, self.seq, 99)

        def step() -> None:
            out = ogpt.train_step(state["params"], ids, targets, cfg, state["state"])
            state["params"], state["state"] = out["params"], out["state"]

        return step, batch * self.seq, (
            f"{batch} x {self.seq} tokens of the workload (full model), float32 NumPy "
            f"restatement of the reference step, {threads} BLAS threads")


class MHAWorkload(Workload):
    SHAPE = (16, 8, 512, 64)

    def __init__(self) -> None:
        super().__init__("mha", "causal MHA fwd+bwd calls/s", "calls/s", 1,
                         "fused causal multi-head attention forward + backward alone: Q, K, V, "
                         "dO (16, 8, 512, 64) ~ N(0, 1); outputs dQ, dK, dV",
                         {"shape": list(self.SHAPE), "causal": True})

    def flops(self) -> float:
        b, h, t, d = self.SHAPE
        return 14.0 * b * h * t * t * d / 2  # fwd 4 + bwd 10 (incl. recompute), causal half

    def build(self, tg, device, rank, reducer_cls) -> Built:
        import numpy as np

        rng = np.random.default_rng(77 + rank)
        arrays = [rng.standard_normal(self.SHAPE).astype(np.float32) for _ in range(4)]

        def step(q, k, v, do):
            q, k, v = (tg.Tensor(a, requires_grad=True) if not isinstance(a, tg.Tensor) or
                       not a.requires_grad else a for a in (q, k, v))
            o = tg.nn.functional.scaled_dot_product_attention(q, k, v, causal=True)
            return tg.autograd.grad(o, [q, k, v], grad_outputs=do)

        dev = tuple(tg.Tensor(a, requires_grad=i < 3) for i, a in enumerate(arrays))
        nbytes = arrays[0].nbytes
        return Built(step, dev, _pinned(device, arrays), 4 * nbytes, 3 * nbytes)

    def cpu_step(self, threads: int):
        import numpy as np

        from oracle import ops as O

        b, h, t, d = self.SHAPE
        rng = np.random.default_rng(5)
        q, k, v, do = (rng.standard_normal((1, h, t, d)).astype(np.float32) for _ in range(4))

        def step() -> None:
            o, p = O.attention_forward(q, k, v, True)
            O.attention_backward(do, q, k, v, p)

        return step, 1.0 / b, (f"1 of the 16 batch entries (8 heads x 512 x 64), float32 NumPy "
                               f"restatement of the reference's attention VJP, {threads} BLAS "
                               "threads; calls/s scaled by 1/16")


class CNNWorkload(Workload):
    def __init__(self) -> None:
        super().__init__("cnn", "CNN fwd+bwd+AdamW samples/s", "samples/s", 256,
                         "CNN train step: Conv2d 3->32 3x3 pad 1 + BatchNorm2d + ReLU + "
                         "MaxPool2d 2, Conv2d 32->64 same, Flatten, Linear 16384->4; 256 images "
                         "3x64x64 ~ N(0,1), 4 classes; cross entropy; AdamW",
                         {"global_batch": 256, "image": [3, 64, 64]})

    def flops(self) -> float:
        from oracle import cnn as ocnn

        return ocnn.step_flops(ocnn.Config(), 256)

    def build(self, tg, device, rank, reducer_cls) -> Built:
        import numpy as np

        from oracle import cnn as ocnn

        cfg = ocnn.Config()
        nn = tg.nn
        model = nn.Sequential(
            nn.Conv2d(3, 32, 3, padding=1), nn.BatchNorm2d(32), nn.ReLU(), nn.MaxPool2d(2),
            nn.Conv2d(32, 64, 3, padding=1), nn.BatchNorm2d(64), nn.ReLU(), nn.MaxPool2d(2),
            nn.Flatten(), nn.Linear(64 * 16 * 16, 4))
        model.load_state_dict(ocnn.init_params(cfg, 3) | ocnn.init_buffers(cfg))
        params = list(model.parameters())
        reducer = reducer_cls(params) if reducer_cls else None
        step = _train_step(tg, model, params, tg.cross_entropy, reducer, None)
        x, labels = ocnn.synthetic_batch(cfg, 256, 100 + rank)
        x = x.astype(np.float32)
        return Built(step, (tg.Tensor(x), tg.Tensor(labels)), _pinned(device, (x, labels)),
                     x.nbytes + labels.nbytes, 4, params)

    def cpu_step(self, threads: int):
        import numpy as np

        from oracle import cnn as ocnn

        cfg = ocnn.Config()
        batch = 16
        params = {k: v.astype(np.float32) for k, v in ocnn.init_params(cfg, 3).items()}
        bufs = {k: v.astype(np.float32) for k, v in ocnn.init_buffers(cfg).items()}
        x, labels = ocnn.synthetic_batch(cfg, batch, 7)
        x = x.astype(np.float32)
        state = {"params": params, "state": None}

        def step() -> None:
            out = ocnn.train_step(state["params"], bufs, x, labels, state["state"])
            state["params"], state["state"] = out["params"], out["state"]

        return step, batch, (f"{batch} of the 256 images, float32 NumPy restatement of the "
                             f"reference step, {threads} BLAS threads")


class RNNWorkload(Workload):
    def __init__(self, cell: str) -> None:
        super().__init__(cell, f"{cell.upper()} BPTT fwd+bwd+AdamW samples/s", "samples/s",
                         512, f"{cell.upper()} adding-problem train step: T 100, batch 512, "
                         "input 2 (values U[0,1], markers {0,1}), hidden 512, Linear 512->1 on "
                         "the last state, MSE, full BPTT, AdamW",
                         {"global_batch": 512, "seq_len": 100, "hidden": 512})
        self.cell = cell

    def flops(self) -> float:
        from oracle import rnn as ornn

        return ornn.step_flops(ornn.Config(cell=self.cell), 512)

    def build(self, tg, device, rank, reducer_cls) -> Built:
        import numpy as np

        from oracle import rnn as ornn

        cfg = ornn.Config(cell=self.cell)
        cell_cls = tg.nn.LSTM if self.cell == "lstm" else tg.nn.GRU

        class Regressor(tg.nn.Module):
            def __init__(self) -> None:
                super().__init__()
                self.rnn = cell_cls(2, 512)
                self.head = tg.nn.Linear(512, 1)

            def forward(self, x):
                output, _ = self.rnn(x)
                return self.head(output[-1])

        model = Regressor()
        model.load_state_dict(ornn.init_params(cfg, 9))
        params = list(model.parameters())
        reducer = reducer_cls(params) if reducer_cls else None
        step = _train_step(tg, model, params, tg.mse_loss, reducer, None)
        x, y = ornn.synthetic_batch(cfg, 512, 200 + rank)
        x, y = x.astype(np.float32), y.astype(np.float32)
        return Built(step, (tg.Tensor(x), tg.Tensor(y)), _pinned(device, (x, y)),
                     x.nbytes + y.nbytes, 4, params)

    def cpu_step(self, threads: int):
        import numpy as np

        from oracle import rnn as ornn

        cfg = ornn.Config(cell=self.cell)
        batch = 32
        params = {k: v.astype(np.float32) for k, v in ornn.init_params(cfg, 9).items()}
        x, y = ornn.synthetic_batch(cfg, batch, 3)
        x, y = x.astype(np.float32), y.astype(np.float32)
        state = {"params": params, "state": None}

        def step() -> None:
            out = ornn.train_step(state["params"], cfg, x, y, state["state"])
            state["params"], state["state"] = out["params"], out["state"]

        return step, batch, (f"{batch} of the 512 sequences (T 100, hidden 512), float32 NumPy "
                             f"restatement of the reference step, {threads} BLAS threads")


WORKLOADS: dict[str, Workload] = {
    "gpt2": GPTWorkload(
        "gpt2", dict(vocab_size=50304, block_size=1024, n_layer=12, n_head=12, n_embd=768), 8,
        1024, "GPT-2-small-shape train step: 12 layers, d_model 768, 12 heads, block 1024, "
              "vocab 50304, tied head; micro-batch 8 x 1024 tokens per GPU; AdamW lr 3e-4 wd "
              "1e-4, clip 1.0"),
    "char_gpt": GPTWorkload(
        "char_gpt", dict(vocab_size=65, block_size=128, n_layer=4, n_head=4, n_embd=128), 32,
        128, "char-level GPT train step: 4 pre-LN layers, d_model 128, 4 heads, block 128, "
             "vocab 65, batch 32; AdamW lr 3e-4 wd 1e-4, clip 1.0"),
    "mha": MHAWorkload(),
    "cnn": CNNWorkload(),
    "lstm": RNNWorkload("lstm"),
    "gru": RNNWorkload("gru"),
}


# ----------------------------------------------------------------------------- CPU legs
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


def cpu_measure(wl: Workload, steps: int, warmup: int, budget_s: float,
                threads: int | None = None) -> tuple[float, int, str, int, float, float]:
    """Units/s of the CPU step on a bounded sample with ``threads`` BLAS threads (default: all
    host cores); also the timed steps, the sample's units and its median seconds per step."""
    from threadpoolctl import threadpool_limits

    threads = threads or os.cpu_count() or 1
    with threadpool_limits(threads):
        step, units, sample = wl.cpu_step(threads)
        for _ in range(warmup):
            step()  # allocator and BLAS warm-up
        sec, n = time_cpu(step, steps, budget_s)
    return units / sec, n, sample, threads, units, sec


def cpu_baseline(wl: Workload, budget_s: float = 30.0) -> dict:
    value, n, sample, threads, _, _ = cpu_measure(wl, 3, 1, budget_s)
    return {"value": value, "unit": wl.unit, "cores": threads, "kind": "port",
            "sample": f"{sample}; median of {n} steps after 1 warm-up"}


def run_reference(args: argparse.Namespace, wl: Workload) -> None:
    """The reference arm: the float32 NumPy restatement of the reference's step (the oracle
    port; the reference itself is a Python package that is not installed on the GPU host) on
    a bounded sample of the workload, timed with every host core and with one BLAS thread
    (the reference's recommended setting); ``value`` is the faster of the two. ``steps`` and
    ``ms_per_step`` describe the sample steps actually timed; the full step's time follows
    from them by the ratio of units and is given as a named extrapolation."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    warm = 1 if args.warmup > 0 else 0
    legs = {}
    # The one-thread leg follows the warmed-up all-cores leg (same process, same sample), so
    # it takes no warm-up step of its own.
    for label, threads, budget, w in (("all_cores", None, 60.0, warm), ("one_thread", 1, 45.0, 0)):
        value, n, sample, used, units, sec = cpu_measure(wl, args.steps, w, budget, threads)
        legs[label] = {"value": value, "threads": used, "steps": n, "ms_per_sample_step": 1e3 * sec,
                       "sample_units": units}
    best = max(legs.values(), key=lambda leg: leg["value"])
    value = best["value"]
    print(json.dumps({
        "impl": "reference", "metric": wl.metric, "value": value, "unit": wl.unit,
        "n_gpus": args.gpus, "steps": best["steps"], "warmup": warm,
        "ms_per_step": best["ms_per_sample_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl.description, **wl.config, "parallelism": "host cores",
                   "sample": sample, "timed_step": "one sample step (see cpu_baseline)"},
        "extrapolated_ms_per_full_step": 1e3 * wl.units_per_step / value,
        "blas_threads": {k: {kk: vv for kk, vv in v.items()} for k, v in legs.items()},
        "cpu_baseline": {"value": value, "unit": wl.unit, "cores": best["threads"],
                         "kind": "port",
                         "sample": f"{sample}; median of {best['steps']} steps"},
        "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- clocks
CLOCK_REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
                 ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
                 ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
                 ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))


def sample_clocks(uuid: str, out_path: str, period: float = 0.005) -> None:
    """Clock sampler process: every ``period`` s append ``monotonic time, SM MHz, max SM MHz,
    clock-event reason bits`` of the GPU ``uuid`` to ``out_path`` (NVML, the fields of
    ``nvidia-smi --query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.*``) until killed.
    Reading them changes no setting of the GPU."""
    import pynvml as nv

    nv.nvmlInit()
    h = nv.nvmlDeviceGetHandleByUUID(uuid)
    mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
    with open(out_path, "w") as f:
        while True:
            sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            f.write(f"{time.monotonic()},{sm},{mx},{bits}\n")
            f.flush()
            time.sleep(period)


class ClockSampler:
    """Runs ``sample_clocks`` in a child process (no contention with the launching thread)
    and summarises the samples taken between ``begin()`` and ``end()``."""

    def __init__(self, local_index: int) -> None:
        import tempfile

        self.proc = None
        self.error = None
        self.t0 = self.t1 = 0.0
        try:
            import torch

            uuid = f"GPU-{torch.cuda.get_device_properties(local_index).uuid}"
        except Exception as exc:  # noqa: BLE001 - no UUID: no sampling, said in the line
            self.error = f"no GPU UUID: {type(exc).__name__}"
            return
        fd, self.path = tempfile.mkstemp(suffix=".clocks")
        os.close(fd)
        import subprocess

        self.proc = subprocess.Popen(
            [sys.executable, os.path.abspath(__file__), "--sample-clocks", uuid, self.path],
            stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        deadline = time.monotonic() + 20.0
        while time.monotonic() < deadline and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.01)
        if self.proc.poll() is not None:
            self.error = "nvml sampler exited"

    def begin(self) -> None:
        self.t0 = time.monotonic()

    def end(self) -> None:
        self.t1 = time.monotonic()

    def stop(self) -> dict:
        if self.proc is None or self.error:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.error], "samples": 0}
        time.sleep(0.02)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = line.strip().split(",")
                if len(parts) == 4:
                    rows.append((float(parts[0]), float(parts[1]), float(parts[2]),
                                 int(parts[3])))
        os.unlink(self.path)
        inside = [r for r in rows if self.t0 <= r[0] <= self.t1]
        if not inside:  # a timed region shorter than one period: the nearest sample after it
            inside = [r for r in rows if r[0] >= self.t1][:1]
        import pynvml as nv

        reasons = sorted({name for *_, bits in inside for name, const in CLOCK_REASONS
                          if bits & int(getattr(nv, const))})
        return {"sm_mhz": statistics.median(r[1] for r in inside) if inside else None,
                "sm_max_mhz": max(r[2] for r in inside) if inside else None,
                "reasons": reasons, "samples": len(inside),
                "source": "nvml every 5 ms during the timed steps"}


# ----------------------------------------------------------------------------- our arm
def _hbm_cases(wl: Workload, device, lib) -> list:
    """The workload's HBM-bound kernels at the step's shapes, each as (name, algorithmic bytes
    per launch, a list of argument sets (one per rotating buffer set), a launcher). The
    algorithmic bytes are the minimum a launch must move: every input read once, every output
    written once."""
    import ctypes

    import numpy as np

    f4 = 4
    st = device.stream()
    rng = np.random.default_rng(7)
    zeros = lambda shape, dt=np.float32: _zeroed(device, lib, shape, dt)  # noqa: E731

    def rnd(shape):
        return device.from_numpy(rng.standard_normal(shape).astype(np.float32))

    def sets(per_set_bytes: int, make) -> list:
        # Enough buffer sets that consecutive launches do not find their inputs in the L2.
        return [make() for _ in range(max(2, -(-(384 << 20) // max(per_set_bytes, 1))))]

    cases = []
    if isinstance(wl, GPTWorkload):
        n, d, v = wl.batch * wl.seq, wl.cfg["n_embd"], wl.cfg["vocab_size"]
        f = 4 * d
        w, b = rnd((d,)), rnd((d,))
        scratch = zeros((lib.tg_layer_norm_scratch_bytes(0, n, d) // 4 + 1,))
        gw, gb = zeros((d,)), zeros((d,))

        def ln_set():
            return dict(x=rnd((n, d)), y=zeros((n, d)), g=rnd((n, d)), gx=zeros((n, d)),
                        mean=zeros((n,)), rstd=zeros((n,)))

        ln = sets(4 * n * d * f4, ln_set)
        for a in ln:
            lib.tg_layer_norm_forward(0, a["x"].ptr, w.ptr, b.ptr, a["y"].ptr, a["mean"].ptr,
                                      a["rstd"].ptr, n, d, 1e-5, st)
        cases.append(("ln_fwd (layer norm forward)", 2 * n * d * f4, ln, lambda a: lib.tg_layer_norm_forward(
            0, a["x"].ptr, w.ptr, b.ptr, a["y"].ptr, a["mean"].ptr, a["rstd"].ptr, n, d, 1e-5, st)))
        cases.append(("ln_bwd (layer norm VJP: gx, gw, gb)", 3 * n * d * f4, ln,
                      lambda a: lib.tg_layer_norm_backward(
                          0, a["g"].ptr, a["x"].ptr, w.ptr, a["mean"].ptr, a["rstd"].ptr,
                          a["gx"].ptr, gw.ptr, gb.ptr, n, d, 7, scratch.ptr, st)))
        ge = sets(3 * n * f * f4, lambda: dict(x=rnd((n, f)), y=zeros((n, f)), g=rnd((n, f))))
        cases.append(("gelu_fwd", 2 * n * f * f4, ge,
                      lambda a: lib.tg_gelu_forward(0, n * f, a["x"].ptr, a["y"].ptr, st)))
        cases.append(("gelu_bwd", 3 * n * f * f4, ge,
                      lambda a: lib.tg_gelu_backward(0, n * f, a["g"].ptr, a["x"].ptr,
                                                     a["y"].ptr, st)))
        logits, grad = zeros((n, v)), zeros((n, v))
        tgt = device.from_numpy(rng.integers(0, v, size=n, dtype=np.int64))
        lse, rows, out = zeros((n,)), zeros((n,)), zeros((1,))
        nvalid, bad = zeros((1,), np.int64), zeros((1,), np.int32)
        one = device.from_numpy(np.ones(1, np.float32))
        ce = [dict()]
        cases.append(("ce_fwd (cross entropy, online log-sum-exp)", n * v * f4, ce,
                      lambda a: lib.tg_cross_entropy_forward(
                          0, logits.ptr, tgt.ptr, lse.ptr, rows.ptr, out.ptr, n, v, -100, 0,
                          nvalid.ptr, bad.ptr, st)))
        cases.append(("ce_bwd (softmax - onehot)", 2 * n * v * f4, ce,
                      lambda a: lib.tg_cross_entropy_backward(
                          0, logits.ptr, tgt.ptr, lse.ptr, one.ptr, nvalid.ptr, grad.ptr, n, v,
                          -100, 0, st)))
    elif isinstance(wl, CNNWorkload):
        from tensorgrad_b200._lib import ConvShape

        n, c, hw = 256, 32, 64 * 64
        w, b = rnd((c,)), rnd((c,))
        mean, rstd, rm, rv = zeros((c,)), zeros((c,)), zeros((c,)), zeros((c,))
        gw, gb = zeros((c,)), zeros((c,))
        scratch = zeros((lib.tg_batch_norm_scratch_bytes(0, n, c, hw) // 4 + 1,))
        bn = sets(4 * n * c * hw * f4, lambda: dict(x=rnd((n, c, hw)), y=zeros((n, c, hw)),
                                                    g=rnd((n, c, hw)), gx=zeros((n, c, hw))))
        cases.append(("bn_fwd (batch norm: statistics + apply)", 2 * n * c * hw * f4, bn,
                      lambda a: lib.tg_batch_norm_forward(
                          0, n, c, hw, a["x"].ptr, w.ptr, b.ptr, a["y"].ptr, mean.ptr, rstd.ptr,
                          rm.ptr, rv.ptr, 0.1, 1e-5, scratch.ptr, st)))
        cases.append(("bn_bwd (batch norm VJP: gx, gw, gb)", 3 * n * c * hw * f4, bn,
                      lambda a: lib.tg_batch_norm_backward(
                          0, n, c, hw, a["g"].ptr, a["x"].ptr, w.ptr, mean.ptr, rstd.ptr,
                          a["gx"].ptr, gw.ptr, gb.ptr, scratch.ptr, st)))
        shp = ConvShape(n=n, c=c, h=64, w=64, c_out=c, kh=2, kw=2, sh=2, sw=2, ph=0, pw=0,
                        oh=32, ow=32)
        q = n * c * 32 * 32
        mp = sets(5 * q * f4, lambda: dict(x=rnd((n, c, 64, 64)), y=zeros((n, c, 32, 32)),
                                           arg=zeros((q,), np.uint8), g=rnd((n, c, 32, 32)),
                                           gx=zeros((n, c, 64, 64))))
        for a in mp:
            lib.tg_max_pool2d_forward(0, ctypes.byref(shp), a["x"].ptr, a["y"].ptr, a["arg"].ptr,
                                      st)
        cases.append(("maxpool_fwd (2x2: y + winner byte)", 4 * q * f4 + q * f4 + q, mp,
                      lambda a: lib.tg_max_pool2d_forward(0, ctypes.byref(shp), a["x"].ptr,
                                                          a["y"].ptr, a["arg"].ptr, st)))
        cases.append(("maxpool_bwd (2x2 gather)", q * f4 + q + 4 * q * f4, mp,
                      lambda a: lib.tg_max_pool2d_backward(0, ctypes.byref(shp), a["g"].ptr,
                                                           a["arg"].ptr, a["gx"].ptr, st)))
    return cases


def _zeroed(device, lib, shape, dt):
    a = device.empty(shape, dt)
    lib.tg_memset_zero(a.ptr, a.nbytes, device.stream())
    return a


def hbm_kernels(wl: Workload, built: Built, reps: int = 20) -> list:
    """Each HBM-bound kernel of the step, launched alone at the step's shapes through the C ABI
    and timed with CUDA events over ``reps`` launches that rotate over buffer sets larger than
    the L2 (so the inputs come from HBM): algorithmic bytes per launch / mean duration,
    against the measured copy bandwidth. AdamW (clip fused) and the clip norm run over a
    parameter arena the size of the model's."""
    import torch

    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import lib

    hbm = float(peaks().get("hbm_gbs", 6650.0))
    cases = _hbm_cases(wl, device, lib)
    nparam = sum(int(p.size) for p in built.params)
    if nparam:
        import ctypes

        import numpy as np

        z = lambda: _zeroed(device, lib, (nparam,), np.float32)  # noqa: E731
        p, g, m, v = z(), z(), z(), z()
        total = _zeroed(device, lib, (1,), np.float64)
        scr = _zeroed(device, lib, (lib.tg_sumsq_scratch_bytes(1) // 4 + 1,), np.float32)
        ptrs, nums = (ctypes.c_void_p * 1)(g.ptr), (ctypes.c_int64 * 1)(nparam)
        st = device.stream()
        cases.append(("adam_flat_vec4 (AdamW with the clip factor fused)", 28 * nparam, [{}],
                      lambda a: lib.tg_adam_update_clipped(
                          0, nparam, p.ptr, g.ptr, m.ptr, v.ptr, 3e-4, 0.9, 0.999, 1e-8, 1e-4, 2,
                          1, total.ptr, 1.0, 1e-6, st)))
        cases.append(("sumsq (clip_grad_norm_ total, float64)", 4 * nparam, [{}],
                      lambda a: lib.tg_sumsq_multi(0, 1, ptrs, nums, total.ptr, scr.ptr, st)))
    out = []
    for name, nbytes, arg_sets, launch in cases:
        for a in arg_sets[:2]:
            launch(a)
        device.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(reps):
            rc = launch(arg_sets[i % len(arg_sets)])
            if rc:
                raise RuntimeError(f"{name}: status {rc}")
        stop.record()
        stop.synchronize()
        us = 1e3 * start.elapsed_time(stop) / reps
        gbs = nbytes / (us * 1e-6) / 1e9
        out.append({"kernel": name, "bytes_per_launch": int(nbytes), "us_per_launch": us,
                    "achieved_gbs": gbs, "frac": gbs / hbm})
    return out


def run_ours(args: argparse.Namespace, wl: Workload) -> None:
    import ctypes

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
    # The attention op alone has no parameters: N GPUs run N replicas.
    reducer_cls = GradientAllReduce if world > 1 and wl.name != "mha" else None
    built = wl.build(tg, device, rank, reducer_cls)
    results: list = []

    def timed(k: int, fn, sampler: ClockSampler | None = None) -> float:
        barrier()
        tg.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if sampler is not None:
            sampler.begin()
        start.record()
        for _ in range(k):
            fn()
        stop.record()
        stop.synchronize()
        if sampler is not None:
            sampler.end()
        barrier()
        return max_over_ranks(start.elapsed_time(stop) / 1e3)

    # Device-resident inputs: the value line.
    clocks = ClockSampler(local)
    for _ in range(args.warmup):
        built.step(*built.dev_inputs)
    launches0 = int(lib.tg_launch_count())
    fallbacks0 = int(lib.tg_gemm_fallback_count())
    sec = timed(args.steps, lambda: built.step(*built.dev_inputs), clocks)
    launches = int(lib.tg_launch_count()) - launches0
    fallbacks = int(lib.tg_gemm_fallback_count()) - fallbacks0
    clock = clocks.stop()
    # The roofline pass: the same steps again with every tensor-core GEMM bracketed by CUDA
    # events (kept out of the value pass, whose launch rate they would slow).
    lib.tg_gemm_profile(1)
    timed(args.steps, lambda: built.step(*built.dev_inputs))
    lib.tg_gemm_profile(0)
    gms, gl, gfl = ctypes.c_double(), ctypes.c_int64(), ctypes.c_double()
    lib.tg_gemm_profile_read(ctypes.byref(gms), ctypes.byref(gl), ctypes.byref(gfl))

    # End to end: pinned host inputs uploaded inside the step, every step's result copied
    # back to page-locked host memory inside the timed region (without blocking the host).
    reader = _AsyncReadback(lib, device)

    def e2e_step():
        reader.issue(built.step(*built.pinned_inputs))

    for _ in range(args.warmup):
        e2e_step()
    sec_e2e = timed(args.steps, e2e_step)
    results.append(reader.value())

    units = wl.units_per_step * world
    pk = peaks()
    achieved = gfl.value / (gms.value / 1e3) / 1e12 if gms.value > 0 else 0.0
    peak = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops")))
    last = results[-1] if results and not isinstance(results[-1], list) else None
    out = {
        "metric": wl.metric,
        "value": units * args.steps / sec,
        "unit": wl.unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * sec / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic seeded inputs of the configuration's shapes; seeded weights",
        "config": {"workload": wl.description, **wl.config,
                   "parallelism": (f"dp{world}" if reducer_cls or world == 1 else
                                   f"{world} replicas"),
                   "matmul": "tcgen05 kind::tf32 with a 3xTF32 split (fp32-level accuracy)",
                   "l2": "no flush: every step streams its activations and parameters; the "
                         "GEMM operands of the timed steps exceed the 126 MB L2 except for the "
                         "small configurations, whose timings include L2 reuse"},
        "roofline": {
            "kernel": "tensor-core GEMM (gemm_tc_kernel, 3xTF32)",
            "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak if peak else None,
            # DRAM bytes per GEMM launch over one step, from an ncu capture of that step's
            # GEMM launches (the 12-layer GPT-2 workload only).
            "traffic": GEMM_TRAFFIC_PER_LAUNCH.get(wl.name) if not (args.layers or args.batch)
            else None,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum over the GEMM "
                              "launches of one step, per launch" if wl.name in
                              GEMM_TRAFFIC_PER_LAUNCH else None,
            "peak_source": f"{pk['source']} bf16_tflops_sustained (dense bf16 cuBLAS)",
            "launches": gl.value, "device_ms_per_step": gms.value / args.steps,
            "tf32_ceiling_frac": achieved / (peak / 2) if peak else None,
            "tf32x3_ceiling_frac": achieved / (peak / 6) if peak else None,
            "step_tflops": wl.flops() * world / (sec / args.steps) / 1e12,
        },
        "clocks": clock,
        "e2e": {"value": units * args.steps / sec_e2e, "unit": wl.unit,
                "h2d_bytes_per_step": int(built.h2d_bytes),
                "d2h_bytes_per_step": int(built.d2h_bytes)},
        "gpu_launches": launches,
        "gemm_fallbacks": fallbacks,  # fp32 products that could not run on the tensor cores
        "final_loss": last,
    }
    if rank == 0 and not args.no_hbm:
        out["hbm_kernels"] = {
            "peak_gbs": float(pk.get("hbm_gbs", 6650.0)),
            "peak_source": f"{pk['source']} hbm_gbs (STREAM-style copy)",
            "method": "each kernel alone at the step's shapes, 20 launches rotating over "
                      "buffer sets larger than the L2, CUDA events; algorithmic bytes",
            "kernels": hbm_kernels(wl, built)}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(wl)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def main() -> None:
    if len(sys.argv) == 4 and sys.argv[1] == "--sample-clocks":
        sample_clocks(sys.argv[2], sys.argv[3])
        return
    args = parse()
    if args.gemm:
        run_gemm(args)
        return
    wl = WORKLOADS[args.workload]
    if (args.layers or args.batch) and isinstance(wl, GPTWorkload):
        cfg = dict(wl.cfg, n_layer=args.layers or wl.cfg["n_layer"])
        batch = args.batch or wl.batch
        wl = GPTWorkload(wl.name, cfg, batch, wl.seq,
                         wl.description + f" [reduced for a capture: {cfg['n_layer']} layers, "
                                          f"micro-batch {batch}]")
    if args.impl == "reference":
        # torchrun sets OMP_NUM_THREADS=1 for N > 1 processes, which OpenBLAS would read when
        # NumPy loads: give the CPU arm every host core whatever the launcher (NumPy is not
        # imported before this point).
        for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS"):
            os.environ[var] = str(os.cpu_count() or 1)
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
