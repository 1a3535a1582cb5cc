"""tensorgrad_b200: tensorgrad's training step on B200 GPUs.

The top-level namespace mirrors ``tensorgrad`` (the reference): the :class:`Tensor` type,
grad-mode switches, factories and the differentiable ops; ``nn``, ``optim`` and ``autograd``
are the same modules. Tensors live in device memory and every op runs hand-written sm_100a
kernels from ``libtgb200.so`` (C ABI in ``include/tgb200.h``); there is no CPU fallback.
"""

from tensorgrad_b200 import autograd, profiler
from tensorgrad_b200._random import get_rng, manual_seed
from tensorgrad_b200.autograd import enable_grad, is_grad_enabled, no_grad
from tensorgrad_b200.device import DeviceArray, set_device, synchronize
from tensorgrad_b200.ops import (
    add, binary_cross_entropy_with_logits, broadcast_to, concat, conv2d, cross_entropy, div,
    dropout, embedding, exp, flatten, gelu, layer_norm, linear, log, log_softmax, logsumexp,
    masked_fill, matmul, max, max_pool2d, mean, min, mse_loss, mul, neg, permute, pow, relu,
    reshape, sigmoid, softmax, sqrt, squeeze, stack, sub, sum, tanh, transpose, unsqueeze, var,
    where,
)
from tensorgrad_b200.tensor import (
    Tensor, arange, full, get_default_dtype, ones, ones_like, rand, randn, set_default_dtype,
    tensor, zeros, zeros_like,
)

from tensorgrad_b200 import func, nn, optim, utils, viz  # noqa: E402  (after the ops they use)

__version__ = "0.1.0"


def _lib_launches() -> int:
    """Kernels launched by libtgb200.so in this process so far."""
    from tensorgrad_b200._lib import lib

    return int(lib.tg_launch_count())

__all__ = [
    "DeviceArray", "Tensor", "__version__", "add", "arange", "autograd",
    "binary_cross_entropy_with_logits", "broadcast_to", "concat", "conv2d", "cross_entropy",
    "div", "dropout", "embedding", "enable_grad", "exp", "flatten", "full", "func", "gelu",
    "get_default_dtype", "get_rng", "is_grad_enabled", "layer_norm", "linear", "log",
    "log_softmax", "logsumexp", "manual_seed", "masked_fill", "matmul", "max", "max_pool2d",
    "mean", "min", "mse_loss", "mul", "neg", "nn", "no_grad", "ones", "ones_like", "optim",
    "permute", "pow", "profiler", "rand", "randn", "relu", "reshape", "set_default_dtype",
    "set_device", "sigmoid", "softmax", "sqrt", "squeeze", "stack", "sub", "sum", "synchronize",
    "tanh", "tensor", "transpose", "unsqueeze", "utils", "var", "viz", "where", "zeros",
    "zeros_like",
]
