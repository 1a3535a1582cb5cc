"""Neural-network building blocks with the reference's API (``tensorgrad.nn``)."""

from tensorgrad_b200.nn import functional, init
from tensorgrad_b200.nn.attention import LayerCache, MultiHeadAttention
from tensorgrad_b200.nn.layers import (
    GELU, MLP, BatchNorm1d, BatchNorm2d, Conv2d, Dropout, Embedding, Flatten, Identity, LayerNorm,
    Linear, MaxPool2d, ReLU, Sequential, Sigmoid, Tanh,
)
from tensorgrad_b200.nn.module import IncompatibleKeys, Module, Parameter
from tensorgrad_b200.nn.recurrent import GRU, LSTM, RNN
from tensorgrad_b200.nn.transformer import GPT, GPTConfig, KVCache, TransformerBlock

__all__ = [
    "GELU", "GPT", "GRU", "LSTM", "MLP", "BatchNorm1d", "BatchNorm2d", "Conv2d", "Dropout", "Embedding",
    "Flatten", "GPTConfig", "Identity", "IncompatibleKeys", "KVCache", "LayerCache", "LayerNorm",
    "Linear", "MaxPool2d",
    "Module", "MultiHeadAttention", "Parameter", "RNN", "ReLU", "Sequential", "Sigmoid", "Tanh",
    "TransformerBlock", "functional", "init",
]
