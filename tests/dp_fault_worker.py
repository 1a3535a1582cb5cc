"""One rank of the departure test (launched by tests/test_gpu_dp.py through
torch.distributed.run on 2 GPUs): one data-parallel step on both ranks, then rank 1 announces
that it leaves (between steps, nothing in flight) and exits; rank 0's next step must raise
CollectiveError from the reducer's peer check, before it launches a collective, and its GPU
must still work afterwards. Each rank writes a one-line report."""

from __future__ import annotations

import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main(out_dir: str) -> None:
    import torch.distributed as dist

    import tensorgrad_b200 as tg
    from oracle import gpt as ogpt
    from tensorgrad_b200 import distributed
    from tensorgrad_b200.distributed import CollectiveError, GradientAllReduce
    from tests.dp_spec import DP_SPEC

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    # The process group only bootstraps (store, unique id); gradients go over NCCL.
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=20))
    tg.set_device(local)
    s = DP_SPEC
    cfg = s["cfg"]
    model = tg.nn.GPT(tg.nn.GPTConfig(vocab_size=cfg.vocab_size, block_size=cfg.block_size,
                                      n_layer=cfg.n_layer, n_head=cfg.n_head,
                                      n_embd=cfg.n_embd, dropout=0.0))
    params = list(model.parameters())
    reducer = GradientAllReduce(params, bucket_bytes=s["bucket_bytes"], deadline_s=20.0)
    per = s["batch"] // world
    mine = slice(rank * per, (rank + 1) * per)
    report = []

    def step(seed: int) -> None:
        ids, targets = ogpt.synthetic_batch(cfg, s["batch"], s["seq"], seed)
        for p in params:
            p.grad = None
        tg.cross_entropy(model(ids[mine]), targets[mine]).backward()
        reducer.reduce()
        tg.synchronize()

    step(s["seed"])
    report.append(f"step1=ok norm={float(np.linalg.norm(params[0].grad.numpy())):.6g}")
    store = dist.distributed_c10d._get_default_store()
    if rank == 1:
        reducer.leave()
        reducer.close(abort=True)
        report.append("left")
    else:
        store.wait([distributed._LEFT.format(1)], datetime.timedelta(seconds=20))
        try:
            step(s["seed"] + 1)
            report.append("step2=ok")
        except CollectiveError as exc:
            report.append(f"step2={type(exc).__name__}")
        reducer.close(abort=True)
        x = tg.Tensor(np.arange(8, dtype=np.float32))
        report.append(f"device_after={float((x * 2.0).sum().item()):.1f}")
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(" ".join(report) + "\n")
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
