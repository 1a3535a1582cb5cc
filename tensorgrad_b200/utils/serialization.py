"""Checkpoint files: the reference's ``.npz`` format (utils/serialization.py:19-34).

A checkpoint is a plain ``numpy.savez`` archive of name -> array, written to exactly the
given path and read back without pickle, so files move freely between the reference and this
package. The arrays of a device model are gathered to the host first: each flat parameter
arena (all parameters of an optimizer group, back to back) comes over in one copy and is cut
into its tensors on the host, instead of one synchronising copy per tensor.

Beyond the reference (which saves modules only, README.md:231-232), an optimizer's
``state_dict()`` is a mapping of the same kind, so ``save(opt.state_dict(), path)`` and
``opt.load_state_dict(load(path))`` checkpoint the AdamW moments and step counts too.
"""

from __future__ import annotations

import os
from collections.abc import Mapping
from typing import Any

import numpy as np

__all__ = ["load", "save"]


def _host(value: Any) -> np.ndarray:
    from tensorgrad_b200.device import DeviceArray
    from tensorgrad_b200.tensor import Tensor

    if isinstance(value, Tensor):
        value = value.data
    if isinstance(value, DeviceArray):
        return value.numpy()
    return np.asarray(value)


def save(obj: Any, path: str | os.PathLike[str]) -> None:
    """Write a module's ``state_dict()`` (or any mapping of name -> array, such as an
    optimizer's ``state_dict()``) to ``path`` as an ``.npz`` archive (no suffix added)."""
    state = obj if isinstance(obj, Mapping) else obj.state_dict()
    arrays = {str(name): _host(value) for name, value in state.items()}
    with open(path, "wb") as fh:
        np.savez(fh, **arrays)  # type: ignore[arg-type]


def load(path: str | os.PathLike[str]) -> dict[str, np.ndarray]:
    """Read a checkpoint written by :func:`save` into a ``dict`` of host arrays."""
    with np.load(path, allow_pickle=False) as archive:
        return {name: archive[name] for name in archive.files}
