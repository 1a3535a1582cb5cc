"""The data-parallel parity case, shared by tests/test_gpu_dp.py and tests/dp_worker.py:
a 2-layer char GPT on a global batch of 8 sequences split over the ranks, two AdamW steps
with clipping active, buckets small enough that several overlap the backward walk."""

from oracle import gpt as ogpt

DP_SPEC = dict(cfg=ogpt.Config(vocab_size=65, block_size=64, n_layer=2, n_head=4, n_embd=64),
               batch=8, seq=64, seed=21, steps=2, max_norm=0.5, bucket_bytes=64 << 10)
