"""Functional interface (``import tensorgrad_b200.nn.functional as F``), as the reference's."""

from tensorgrad_b200.ops import (  # noqa: F401
    batch_norm, binary_cross_entropy_with_logits, conv2d, cross_entropy, dropout, embedding,
    gelu, gru, layer_norm, linear, log_softmax, lstm, max_pool2d, mse_loss, relu, rnn, sigmoid,
    softmax, tanh,
)
from tensorgrad_b200.ops.attention import (  # noqa: F401
    packed_self_attention, scaled_dot_product_attention,
)
