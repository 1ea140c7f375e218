"""numpy stand-ins for the ``mlx.nn`` names the reference's dflash.py uses."""
import numpy as np

from . import core as _mx


class Module:
    pass


class Linear(Module):
    def __init__(self, input_dims, output_dims, bias=True):
        assert not bias
        self.weight = np.zeros((output_dims, input_dims), dtype=np.float32)

    def __call__(self, x):
        return np.matmul(x, self.weight.T)


class RMSNorm(Module):
    def __init__(self, dims, eps=1e-5):
        self.weight = np.ones((dims,), dtype=np.float32)
        self.eps = eps

    def __call__(self, x):
        return _mx.fast.rms_norm(x, self.weight, self.eps)


class RoPE(Module):
    def __init__(self, dims, traditional=False, base=10000.0, scale=1.0):
        self.dims, self.traditional, self.base, self.scale = dims, traditional, base, scale


def silu(x):
    return x / (1.0 + np.exp(-x))
