"""SGD with optional (Nesterov) momentum and L2 weight decay (the reference's optim/sgd.py:15-58),
as axpby kernels on the device."""

from __future__ import annotations

from collections.abc import Iterable
from dataclasses import dataclass
from typing import Any

from tensorgrad_b200 import device
from tensorgrad_b200._lib import check, lib
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.optim.optimizer import Optimizer

__all__ = ["SGD"]


@dataclass
class _SGDState:
    momentum_buffer: DeviceArray | None = None


def _axpby(alpha: float, x: DeviceArray, beta: float, y: DeviceArray | None,
           out: DeviceArray) -> DeviceArray:
    check(lib.tg_axpby(dtype_code(x.dtype), x.size, alpha, x.ptr, beta,
                       y.ptr if y is not None else None, out.ptr, device.stream()), "sgd")
    return out


class SGD(Optimizer[_SGDState]):
    """``g += wd p``; ``b = m b + g``; ``d = g + m b`` (Nesterov) or ``b``; ``p -= lr d``."""

    def __init__(self, params: Iterable[Any], lr: float = 1e-2, momentum: float = 0.0,
                 nesterov: bool = False, weight_decay: float = 0.0) -> None:
        if momentum < 0:
            raise ValueError(f"invalid momentum {momentum}")
        if nesterov and momentum == 0:
            raise ValueError("Nesterov momentum requires momentum > 0")
        super().__init__(params, lr, weight_decay)
        self.momentum = momentum
        self.nesterov = nesterov

    def step(self) -> None:
        for group in self.param_groups:
            for p in group.params:
                if p.grad is None:
                    continue
                st = self.state.setdefault(id(p), _SGDState())
                g = p.grad.data if p.grad.dtype == p.dtype else p.grad.data.astype(p.dtype)
                if group.weight_decay:
                    g = _axpby(group.weight_decay, p.data, 1.0, g, device.empty(p.shape, p.dtype))
                if self.momentum:
                    buf = st.momentum_buffer
                    if buf is None:
                        buf = g.copy()
                    else:
                        _axpby(self.momentum, buf, 1.0, g, buf)
                    st.momentum_buffer = buf
                    if self.nesterov:
                        g = _axpby(self.momentum, buf, 1.0, g, device.empty(p.shape, p.dtype))
                    else:
                        g = buf
                _axpby(-group.lr, g, 1.0, p.data, p.data)
