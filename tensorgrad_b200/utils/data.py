"""Mini-batches of in-memory host arrays, uploaded to the device (the reference's
utils/data.py:15-68: same arguments, same order of examples, same batch boundaries).

Each batch is gathered on the host in one indexing pass per array and uploaded with one
asynchronous copy (through the library's reused page-locked staging blocks); labels stay
integer tensors (device-resident targets and ids are accepted by the loss and embedding ops
without a host round trip).
"""

from __future__ import annotations

from collections.abc import Iterator
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200.tensor import Tensor

__all__ = ["DataLoader"]


class DataLoader:
    """Iterate over aligned arrays (same first dimension) in mini-batches of tensors.

    Args:
        *arrays: e.g. inputs and labels.
        batch_size: Examples per batch.
        shuffle: A fresh permutation every epoch, from a generator of its own (``seed``),
            independent of the global one.
        drop_last: Skip a final batch smaller than ``batch_size``.
        seed: Seed of the shuffling generator.
    """

    def __init__(self, *arrays: Any, batch_size: int = 32, shuffle: bool = False,
                 drop_last: bool = False, seed: int | None = None) -> None:
        if not arrays:
            raise ValueError("DataLoader needs at least one array")
        lengths = {len(a) for a in arrays}
        if len(lengths) != 1:
            raise ValueError(f"arrays have different lengths: {sorted(lengths)}")
        if batch_size <= 0:
            raise ValueError("batch_size must be positive")
        self.arrays = tuple(np.asarray(a) for a in arrays)
        self.batch_size, self.shuffle, self.drop_last = batch_size, shuffle, drop_last
        self._rng = np.random.default_rng(seed)

    @property
    def num_examples(self) -> int:
        """Examples per epoch, before batching."""
        return len(self.arrays[0])

    def __len__(self) -> int:
        full, rest = divmod(self.num_examples, self.batch_size)
        return full if self.drop_last or rest == 0 else full + 1

    def batches(self) -> Iterator[np.ndarray]:
        """The example indices of each batch of one epoch (host arrays)."""
        n = self.num_examples
        order = self._rng.permutation(n) if self.shuffle else np.arange(n)
        stop = n - n % self.batch_size if self.drop_last else n
        for start in range(0, stop, self.batch_size):
            yield order[start:start + self.batch_size]

    def __iter__(self) -> Iterator[tuple[Tensor, ...]]:
        for idx in self.batches():
            yield tuple(Tensor._wrap(device.from_numpy(np.take(a, idx, axis=0)))
                        for a in self.arrays)
