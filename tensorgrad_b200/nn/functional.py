"""Functional interface (``import tensorgrad_b200.nn.functional as F``), as the reference's."""

from tensorgrad_b200.ops import (  # noqa: F401
    batch_norm, conv2d, cross_entropy, dropout, embedding, gelu, gru, layer_norm, linear, lstm,
    max_pool2d, mse_loss, relu, sigmoid, tanh,
)
from tensorgrad_b200.ops.attention import (  # noqa: F401
    packed_self_attention, scaled_dot_product_attention,
)
