"""numpy stand-in for the slice of ``mlx.nn`` that the reference's GDN code
touches.  TEST INFRASTRUCTURE ONLY (see core.py)."""
from __future__ import annotations

import numpy as np

from . import core as mx


class Module:
    def __init__(self):
        pass


class Linear(Module):
    def __init__(self, input_dims, output_dims, bias=True):
        super().__init__()
        self.weight = mx.zeros((output_dims, input_dims))
        self.bias = mx.zeros((output_dims,)) if bias else None

    def __call__(self, x):
        y = x @ self.weight.T
        return y + self.bias if self.bias is not None else y


class Embedding(Module):
    def __init__(self, num, dims):
        super().__init__()
        self.weight = mx.zeros((num, dims))


def silu(x):
    return x * mx.sigmoid(x)


def softplus(x):
    return mx.logaddexp(x, 0.0)


def quantize(*a, **kw):
    raise RuntimeError("quantisation is not part of the numpy MLX stand-in")
