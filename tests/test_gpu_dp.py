"""Data parallel on 2 GPUs: two ranks on halves of the global batch, gradients averaged by
the bucketed NCCL all-reduce that overlaps the backward walk, must equal the float64 oracle
run on the whole batch (loss, clip norm, every gradient, post-AdamW parameters) at 1e-4.
Skipped on a single-GPU machine."""

from __future__ import annotations

import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from oracle import gpt as ogpt
from tests.conftest import assert_parity, assert_update_parity, ill_conditioned
from tests.dp_spec import DP_SPEC

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_two_rank_data_parallel_matches_full_batch_oracle(tmp_path):
    out = tmp_path / "dp.npz"
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(_port()), os.path.join(ROOT, "tests", "dp_worker.py"), str(out)]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="0,1")
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    got = dict(np.load(out))
    s = DP_SPEC
    cfg = s["cfg"]
    params, state = ogpt.init_params(cfg, s["seed"]), None
    ill: dict[str, np.ndarray] = {}
    for step in range(1, s["steps"] + 1):
        ids, targets = ogpt.synthetic_batch(cfg, s["batch"], s["seq"], s["seed"] + step)
        ref = ogpt.train_step(params, ids, targets, cfg, state, max_norm=s["max_norm"])
        assert float(got[f"step{step}/loss"]) == pytest.approx(ref["loss"], rel=1e-4)
        assert float(got[f"step{step}/total_norm"]) == pytest.approx(ref["total_norm"], rel=1e-4)
        for n, g in ref["grads"].items():
            assert_parity(got[f"step{step}/grad/{n}"], g, 1e-4, f"step{step} grad {n}")
            mask = ill_conditioned(g, 1e-4)
            ill[n] = mask if n not in ill else (ill[n] | mask)
        for n, p in ref["params"].items():
            assert_update_parity(got[f"step{step}/param/{n}"], p, ill[n], 1e-4,
                                 f"step{step} param {n}")
        # Several buckets, launched from the end of the arena (the backward order).
        order = list(got[f"step{step}/buckets"])
        assert len(order) > 2 and order[0] == max(order)
        params, state = ref["params"], ref["state"]


_NO_NVLS = {"NCCL_NVLS_ENABLE": "0"}


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_departed_rank_raises_before_the_next_exchange(tmp_path):
    cmd = ["timeout", "-k", "30", "180", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(_port()), os.path.join(ROOT, "tests", "dp_fault_worker.py"),
           str(tmp_path)]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="0,1", **_NO_NVLS)
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=240)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    r0 = (tmp_path / "rank0.txt").read_text().split()
    r1 = (tmp_path / "rank1.txt").read_text().split()
    assert r0[:2] == r1[:2] and r0[0] == "step1=ok"  # same averaged gradient on both
    assert r1[2:] == ["left"]
    assert r0[2:] == ["step2=CollectiveError", "device_after=56.0"]


def test_communicator_setup_times_out_without_peers():
    """A two-rank NCCL set-up with no second rank ends in CollectiveTimeout after its
    deadline (the library aborts the half-made communicator); the device still works."""
    code = (
        "import ctypes, time, numpy as np, tensorgrad_b200 as tg\n"
        "from tensorgrad_b200._lib import lib\n"
        "from tensorgrad_b200.distributed import NcclCommunicator, CollectiveTimeout, "
        "_nccl_library\n"
        "tg.set_device(0)\n"
        "assert lib.tg_comm_load((_nccl_library() or '').encode()) == 0\n"
        "uid = ctypes.create_string_buffer(128)\n"
        "assert lib.tg_comm_unique_id(uid, 128) == 0\n"
        "t = time.monotonic()\n"
        "try:\n"
        "    NcclCommunicator(2, 0, uid.raw, timeout_s=3.0)\n"
        "    print('no-timeout')\n"
        "except CollectiveTimeout as e:\n"
        "    print('timeout', round(time.monotonic() - t, 1))\n"
        "x = tg.Tensor(np.arange(8, dtype=np.float32))\n"
        "print('device', float((x * 2.0).sum().item()))\n")
    env = dict(os.environ, **_NO_NVLS)
    res = subprocess.run(["timeout", "-k", "10", "90", sys.executable, "-c", code], cwd=ROOT,
                         env=env, capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    # NCCL writes its own warnings (the aborted set-up) to stdout too.
    mine = [ln for ln in res.stdout.splitlines() if ln.split()[:1] in (["timeout"], ["device"],
                                                                          ["no-timeout"])]
    assert len(mine) == 2, res.stdout[-2000:]
    kind, secs = mine[0].split()
    assert kind == "timeout" and 2.5 <= float(secs) < 30.0
    assert mine[1] == "device 56.0"
