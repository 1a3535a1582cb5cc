"""Adam and AdamW (the reference's optim/adam.py:38-94) as device kernels.

At construction each parameter group is re-homed into a flat arena (parameters and gradient
slots contiguous, 16-byte aligned), and the moments get buffers of the same layout. When
every parameter of a group has its gradient in its slot and all share one step count, the
whole group is ONE ``tg_adam_update`` launch over the flat buffers; otherwise the update is
a multi-tensor launch over the parameters that have gradients, each with its own step count,
exactly the reference's per-parameter semantics.
"""

from __future__ import annotations

from collections.abc import Iterable
from dataclasses import dataclass
from typing import Any

from tensorgrad_b200 import device
from tensorgrad_b200._lib import check, int64_array, lib, ptr_array
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.optim.arena import Arena, arena_of, flatten_parameters
from tensorgrad_b200.optim.optimizer import Optimizer, ParamGroup
from tensorgrad_b200.tensor import Tensor

__all__ = ["Adam", "AdamW"]


@dataclass
class _AdamState:
    exp_avg: DeviceArray
    exp_avg_sq: DeviceArray
    step: int = 0


class Adam(Optimizer[_AdamState]):
    """Adam with bias correction; ``weight_decay`` is L2 added to the gradient."""

    decoupled_weight_decay = False

    def __init__(self, params: Iterable[Any], lr: float = 1e-3,
                 betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0) -> None:
        if not (0.0 <= betas[0] < 1.0 and 0.0 <= betas[1] < 1.0):
            raise ValueError(f"invalid betas {betas}")
        if eps < 0:
            raise ValueError(f"invalid eps {eps}")
        super().__init__(params, lr, weight_decay)
        self.betas = betas
        self.eps = eps
        self._moments: dict[int, tuple[DeviceArray, DeviceArray]] = {}
        for group in self.param_groups:
            for arena in flatten_parameters(group.params):
                if id(arena) not in self._moments:
                    self._moments[id(arena)] = (device.zeros((arena.numel,), arena.dtype),
                                                device.zeros((arena.numel,), arena.dtype))

    def _state_for(self, p: Tensor) -> _AdamState:
        st = self.state.get(id(p))
        if st is None:
            arena: Arena | None = getattr(p, "_arena", None)
            if arena is not None and id(arena) in self._moments and arena.intact():
                m_buf, v_buf = self._moments[id(arena)]
                off = arena.offsets[arena.index[id(p)]]
                st = _AdamState(m_buf.flat_view(off, p.size, p.shape),
                                v_buf.flat_view(off, p.size, p.shape))
            else:
                st = _AdamState(device.zeros(p.shape, p.dtype), device.zeros(p.shape, p.dtype))
            self.state[id(p)] = st
        return st

    def _flat_ok(self, group: ParamGroup) -> Arena | None:
        arena = arena_of(group.params)
        if arena is None or id(arena) not in self._moments:
            return None
        if not (arena.intact() and arena.grads_in_slots()):
            return None
        steps = {self.state[id(p)].step if id(p) in self.state else 0 for p in group.params}
        if len(steps) != 1:
            return None
        m_buf, _ = self._moments[id(arena)]
        for p, off in zip(arena.params, arena.offsets, strict=True):
            st = self.state.get(id(p))
            if st is not None and st.exp_avg.ptr != m_buf.ptr + off * arena.dtype.itemsize:
                return None
        return arena

    def step(self) -> None:
        b1, b2 = self.betas
        for group in self.param_groups:
            wd = group.weight_decay
            arena = self._flat_ok(group)
            if arena is not None:
                states = [self._state_for(p) for p in group.params]
                for st in states:
                    st.step += 1
                m_buf, v_buf = self._moments[id(arena)]
                # A clip rescale left pending by clip_grad_norm_ is applied in the same pass
                # (and stays pending on the gradients themselves).
                clip = arena.pending_clip
                check(lib.tg_adam_update_clipped(
                    dtype_code(arena.dtype), arena.numel, arena.param_buf.ptr,
                    arena.grad_buf.ptr, m_buf.ptr, v_buf.ptr, group.lr, b1, b2, self.eps, wd,
                    states[0].step, int(self.decoupled_weight_decay),
                    clip[0].ptr if clip else None, clip[1] if clip else 0.0,
                    clip[2] if clip else 0.0, device.stream()), "adam step")
                continue
            by_dtype: dict[str, list[tuple[Tensor, DeviceArray, _AdamState]]] = {}
            for p in group.params:
                if p.grad is None:
                    continue
                st = self._state_for(p)
                st.step += 1
                g = p.grad.data if p.grad.dtype == p.dtype else p.grad.data.astype(p.dtype)
                by_dtype.setdefault(str(p.dtype), []).append((p, g, st))
            for items in by_dtype.values():
                code = dtype_code(items[0][0].dtype)
                n = len(items)
                check(lib.tg_adam_update_multi(
                    code, n, ptr_array(p.data.ptr for p, _, _ in items),
                    ptr_array(g.ptr for _, g, _ in items),
                    ptr_array(s.exp_avg.ptr for _, _, s in items),
                    ptr_array(s.exp_avg_sq.ptr for _, _, s in items),
                    int64_array(p.size for p, _, _ in items),
                    int64_array(s.step for _, _, s in items), group.lr, b1, b2, self.eps, wd,
                    int(self.decoupled_weight_decay), None, device.stream()), "adam step")


    # ------------------------------------------------------------------ checkpoints
    # No counterpart in the reference, which cannot save optimizer state (README.md:231-232).
    # Keys: "group.{g}.lr" / "group.{g}.weight_decay", "betas", "eps", and per parameter with
    # state (index i over all groups in order) "state.{i}.step", "state.{i}.exp_avg",
    # "state.{i}.exp_avg_sq". Moments held in an arena come to the host in one copy each.
    def _indexed_params(self) -> list[Tensor]:
        return [p for group in self.param_groups for p in group.params]

    def state_dict(self) -> dict[str, Any]:
        import numpy as np

        out: dict[str, Any] = {"betas": np.asarray(self.betas, np.float64),
                               "eps": np.asarray(self.eps, np.float64)}
        for g, group in enumerate(self.param_groups):
            out[f"group.{g}.lr"] = np.asarray(group.lr, np.float64)
            out[f"group.{g}.weight_decay"] = np.asarray(group.weight_decay, np.float64)
        host_moments: dict[int, tuple[Any, Any]] = {}
        for i, p in enumerate(self._indexed_params()):
            st = self.state.get(id(p))
            if st is None:
                continue
            arena = getattr(p, "_arena", None)
            key = id(arena)
            if arena is not None and key in self._moments and arena.intact():
                if key not in host_moments:
                    host_moments[key] = tuple(b.numpy() for b in self._moments[key])
                m_host, v_host = host_moments[key]
                off = arena.offsets[arena.index[id(p)]]
                m_buf, _ = self._moments[key]
                if st.exp_avg.ptr == m_buf.ptr + off * arena.dtype.itemsize:
                    m = m_host[off:off + p.size].reshape(p.shape).copy()
                    v = v_host[off:off + p.size].reshape(p.shape).copy()
                else:
                    m, v = st.exp_avg.numpy(), st.exp_avg_sq.numpy()
            else:
                m, v = st.exp_avg.numpy(), st.exp_avg_sq.numpy()
            out[f"state.{i}.step"] = np.asarray(st.step, np.int64)
            out[f"state.{i}.exp_avg"] = m
            out[f"state.{i}.exp_avg_sq"] = v
        return out

    def load_state_dict(self, state: Any) -> None:
        """Restore moments, step counts and hyper-parameters saved by :meth:`state_dict`."""
        import numpy as np

        params = self._indexed_params()
        for g, group in enumerate(self.param_groups):
            if f"group.{g}.lr" in state:
                group.lr = float(state[f"group.{g}.lr"])
            if f"group.{g}.weight_decay" in state:
                group.weight_decay = float(state[f"group.{g}.weight_decay"])
        if "betas" in state:
            b = np.asarray(state["betas"], np.float64)
            self.betas = (float(b[0]), float(b[1]))
        if "eps" in state:
            self.eps = float(state["eps"])
        indices = sorted({int(k.split(".")[1]) for k in state if k.startswith("state.")})
        for i in indices:
            if not 0 <= i < len(params):
                raise KeyError(f"optimizer state for parameter {i}, which does not exist")
            p = params[i]
            st = self._state_for(p)
            for name, buf in (("exp_avg", st.exp_avg), ("exp_avg_sq", st.exp_avg_sq)):
                value = np.asarray(state[f"state.{i}.{name}"])
                if value.shape != tuple(p.shape):
                    raise ValueError(f"shape mismatch for 'state.{i}.{name}': expected "
                                     f"{tuple(p.shape)}, got {value.shape}")
                buf[...] = value
            st.step = int(state[f"state.{i}.step"])


class AdamW(Adam):
    """Adam with decoupled weight decay: ``p *= 1 - lr * wd`` before the moment update."""

    decoupled_weight_decay = True

    def __init__(self, params: Iterable[Any], lr: float = 1e-3,
                 betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2) -> None:
        super().__init__(params, lr, betas, eps, weight_decay)
