"""numpy stand-ins for the ``mlx.core`` names the reference's dflash.py uses."""
import types

import numpy as np

float32 = np.float32
float16 = np.float16
float64 = np.float64
int32 = np.int32
Dtype = type(np.dtype(np.float32))


def array(x, dtype=None):
    return np.asarray(x, dtype=dtype)


def concatenate(xs, axis=0):
    return np.concatenate(list(xs), axis=axis)


def repeat(x, repeats, axis):
    # mx.repeat: each slice repeated consecutively (numpy semantics)
    return np.repeat(x, repeats, axis=axis)


def argmax(x, axis=-1):
    # first index of the maximum
    return np.argmax(x, axis=axis)


def argsort(x, axis=-1):
    # ascending; equal keys keep their index order
    return np.argsort(x, axis=axis, kind="stable")


def softmax(x, axis=None):
    x = np.asarray(x)
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def sum(x, axis=None, keepdims=False):  # noqa: A001 - mlx.core.sum
    return np.sum(x, axis=axis, keepdims=keepdims)


def eval(*args):
    return None


def _rms_norm(x, weight, eps):
    xf = x.astype(np.float64) if x.dtype == np.float64 else x.astype(np.float32)
    ms = np.mean(xf * xf, axis=-1, keepdims=True)
    return (xf / np.sqrt(ms + eps) * weight).astype(x.dtype)


def _rope(x, dims, traditional=False, base=10000.0, scale=1.0, offset=0):
    assert not traditional and dims == x.shape[-1]
    half = dims // 2
    inv = (float(base) ** (-2.0 * np.arange(half, dtype=np.float64) / dims)).astype(x.dtype)
    pos = (np.arange(x.shape[-2]) + offset).astype(x.dtype) * np.asarray(scale, dtype=x.dtype)
    ang = pos[:, None] * inv[None, :]
    c, s = np.cos(ang), np.sin(ang)
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1).astype(x.dtype)


def _sdpa(q, k, v, scale, mask=None):
    assert mask is None
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * np.asarray(scale, dtype=q.dtype)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.matmul(p, v).astype(q.dtype)


fast = types.SimpleNamespace(rms_norm=_rms_norm, rope=_rope,
                             scaled_dot_product_attention=_sdpa)
random = types.SimpleNamespace()
