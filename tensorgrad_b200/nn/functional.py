"""Functional interface (``import tensorgrad_b200.nn.functional as F``), as the reference's."""

from tensorgrad_b200.ops import (  # noqa: F401
    batch_norm, cross_entropy, dropout, embedding, gelu, layer_norm, linear, mse_loss, relu,
    sigmoid, tanh,
)
from tensorgrad_b200.ops.attention import (  # noqa: F401
    packed_self_attention, scaled_dot_product_attention,
)
