"""Utilities kept from the reference's ``tensorgrad.utils``: checkpoint files."""

from tensorgrad_b200.utils.serialization import load, save

__all__ = ["load", "save"]
