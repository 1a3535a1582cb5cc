"""Utilities kept from the reference's ``tensorgrad.utils``: data loading, gradient checks,
gradient checkpointing (block recomputation in the backward pass), checkpoint files and host
allocator tuning."""

from tensorgrad_b200.utils.data import DataLoader
from tensorgrad_b200.utils.grad_checkpoint import checkpoint
from tensorgrad_b200.utils.gradcheck import GradcheckError, gradcheck, gradgradcheck, numerical_grad
from tensorgrad_b200.utils.memory import retain_freed_memory
from tensorgrad_b200.utils.serialization import load, save

__all__ = [
    "DataLoader", "GradcheckError", "checkpoint", "gradcheck", "gradgradcheck", "load",
    "numerical_grad", "retain_freed_memory", "save",
]
