"""One rank of the data-parallel parity run (launched by tests/test_gpu_dp.py through
torch.distributed.run): a small GPT on its half of the global batch, gradients averaged by
the bucketed all-reduce, two AdamW steps; rank 0 saves what it saw."""

from __future__ import annotations

import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main(out_path: str) -> None:
    import torch
    import torch.distributed as dist

    import tensorgrad_b200 as tg
    from oracle import gpt as ogpt
    from tensorgrad_b200.distributed import GradientAllReduce
    from tests.dp_spec import DP_SPEC

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", local))
    tg.set_device(local)
    s = DP_SPEC
    cfg = s["cfg"]
    model = tg.nn.GPT(tg.nn.GPTConfig(vocab_size=cfg.vocab_size, block_size=cfg.block_size,
                                      n_layer=cfg.n_layer, n_head=cfg.n_head,
                                      n_embd=cfg.n_embd, dropout=0.0))
    params_np = ogpt.init_params(cfg, s["seed"])
    state = dict(params_np)
    state["head.weight"] = params_np["tok_emb.weight"]
    model.load_state_dict(state)
    names = [n for n, _ in model.named_parameters()]
    params = list(model.parameters())
    opt = tg.optim.AdamW(params, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
    reducer = GradientAllReduce(params, bucket_bytes=s["bucket_bytes"])
    per = s["batch"] // world
    rec: dict[str, np.ndarray] = {}
    for step in range(1, s["steps"] + 1):
        ids, targets = ogpt.synthetic_batch(cfg, s["batch"], s["seq"], s["seed"] + step)
        mine = slice(rank * per, (rank + 1) * per)
        loss = tg.cross_entropy(model(ids[mine]), targets[mine])
        opt.zero_grad()
        loss.backward()
        reducer.reduce()
        total = tg.optim.clip_grad_norm_(params, s["max_norm"])
        lt = torch.tensor([loss.item()], dtype=torch.float64, device="cuda")
        dist.all_reduce(lt)
        rec[f"step{step}/loss"] = np.asarray(lt.item() / world)
        rec[f"step{step}/total_norm"] = np.asarray(total)
        for n, p in zip(names, params, strict=True):
            rec[f"step{step}/grad/{n}"] = p.grad.numpy()
        opt.step()
        for n, p in zip(names, params, strict=True):
            rec[f"step{step}/param/{n}"] = p.numpy()
        rec[f"step{step}/buckets"] = np.asarray(reducer.buckets.last_order)
    reducer.close()
    if rank == 0:
        np.savez(out_path, **rec)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
