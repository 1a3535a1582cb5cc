"""Utilities kept from the reference's ``tensorgrad.utils``: checkpoint files and gradient
checkpointing (block recomputation in the backward pass)."""

from tensorgrad_b200.utils.grad_checkpoint import checkpoint
from tensorgrad_b200.utils.serialization import load, save

__all__ = ["checkpoint", "load", "save"]
