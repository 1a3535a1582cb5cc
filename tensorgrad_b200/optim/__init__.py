"""Optimisers, learning-rate schedules and gradient clipping (the reference's ``optim``)."""

from tensorgrad_b200.optim.adam import Adam, AdamW
from tensorgrad_b200.optim.arena import Arena, flatten_parameters
from tensorgrad_b200.optim.clip import clip_grad_norm_
from tensorgrad_b200.optim.lr_scheduler import CosineWarmupLR, LRScheduler, StepLR
from tensorgrad_b200.optim.optimizer import Optimizer, ParamGroup, ParamGroupSpec
from tensorgrad_b200.optim.sgd import SGD

__all__ = ["SGD", "Adam", "AdamW", "Arena", "CosineWarmupLR", "LRScheduler", "Optimizer",
           "ParamGroup", "ParamGroupSpec", "StepLR", "clip_grad_norm_", "flatten_parameters"]
