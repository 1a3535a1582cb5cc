"""Differentiable ops on device tensors; each records a node whose VJP runs device kernels."""

from tensorgrad_b200 import tensor as _tensor  # noqa: F401  (binds Tensor before the ops)
from tensorgrad_b200.ops.activation import log_softmax, logsumexp, softmax
from tensorgrad_b200.ops.attention import packed_self_attention, scaled_dot_product_attention
from tensorgrad_b200.ops.conv import conv2d, max_pool2d
from tensorgrad_b200.ops.elementwise import (
    add, astype, div, exp, gelu, log, mul, neg, pow, relu, sigmoid, sqrt, sub, tanh,
)
from tensorgrad_b200.ops.layers import batch_norm, dropout, embedding, layer_norm, linear
from tensorgrad_b200.ops.linalg import matmul
from tensorgrad_b200.ops.loss import binary_cross_entropy_with_logits, cross_entropy, mse_loss
from tensorgrad_b200.ops.recurrent import gru, lstm, rnn
from tensorgrad_b200.ops.reduce import max, mean, min, sum, var
from tensorgrad_b200.ops.shape import (
    broadcast_to, concat, flatten, getitem, masked_fill, permute, reshape, squeeze, stack, sum_to,
    transpose, unsqueeze, where,
)

__all__ = [
    "add", "astype", "batch_norm", "binary_cross_entropy_with_logits", "broadcast_to", "concat",
    "conv2d", "cross_entropy", "div", "dropout", "embedding", "exp", "flatten", "gelu", "getitem",
    "gru", "layer_norm", "linear", "log", "log_softmax", "logsumexp", "lstm", "masked_fill",
    "matmul", "max", "max_pool2d", "mean", "min", "mse_loss", "mul", "neg",
    "packed_self_attention", "permute", "pow", "relu", "reshape", "rnn",
    "scaled_dot_product_attention", "sigmoid", "softmax", "sqrt", "squeeze", "stack", "sub",
    "sum", "sum_to", "tanh", "transpose", "unsqueeze", "var", "where",
]
