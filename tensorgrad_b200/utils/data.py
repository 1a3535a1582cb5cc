"""Mini-batches of in-memory host arrays, uploaded to the device (API of the reference's
utils/data.py: the same arguments, example order and batch boundaries).

An epoch is one permutation (or the identity) of the example indices cut into consecutive
slices of ``batch_size``; each batch is gathered on the host, one ``np.take`` per array, and
uploaded with one asynchronous copy through the library's reused page-locked staging
blocks. Integer labels stay int64 tensors, which the loss and embedding ops take on the
device without a host round trip.
"""

from __future__ import annotations

from collections.abc import Iterator
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200.tensor import Tensor

__all__ = ["DataLoader"]


class DataLoader:
    """Aligned arrays (one example per row of each) in mini-batches of device tensors.

    Args:
        *arrays: e.g. inputs and labels, all of one length.
        batch_size: Examples per batch.
        shuffle: A new permutation each epoch, drawn from the loader's own generator
            (seeded by ``seed``, independent of the global generator).
        drop_last: Leave out a last batch shorter than ``batch_size``.
        seed: Seed of that generator.
    """

    def __init__(self, *arrays: Any, batch_size: int = 32, shuffle: bool = False,
                 drop_last: bool = False, seed: int | None = None) -> None:
        if len(arrays) == 0:
            raise ValueError("DataLoader needs at least one array")
        sizes = sorted({len(a) for a in arrays})
        if len(sizes) > 1:
            raise ValueError(f"arrays have different lengths: {sizes}")
        if batch_size < 1:
            raise ValueError("batch_size must be positive")
        self.arrays = tuple(np.asarray(a) for a in arrays)
        self.batch_size = batch_size
        self.shuffle = shuffle
        self.drop_last = drop_last
        self._rng = np.random.default_rng(seed)

    @property
    def num_examples(self) -> int:
        """Examples in one epoch."""
        return self.arrays[0].shape[0]

    def _used(self) -> int:
        """Examples that go into batches (all, or whole batches only with ``drop_last``)."""
        n = self.num_examples
        return n - n % self.batch_size if self.drop_last else n

    def __len__(self) -> int:
        return -(-self._used() // self.batch_size)

    def batches(self) -> Iterator[np.ndarray]:
        """The example indices of each batch of one epoch."""
        n = self.num_examples
        order = self._rng.permutation(n) if self.shuffle else np.arange(n)
        used, size = self._used(), self.batch_size
        for k in range(-(-used // size)):
            yield order[k * size:min((k + 1) * size, used)]

    def __iter__(self) -> Iterator[tuple[Tensor, ...]]:
        for idx in self.batches():
            yield tuple(Tensor._wrap(device.from_numpy(np.take(a, idx, axis=0)))
                        for a in self.arrays)
