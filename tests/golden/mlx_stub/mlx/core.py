"""numpy stand-in for the slice of the ``mlx.core`` API that the reference's
Gated DeltaNet code uses.  TEST INFRASTRUCTURE ONLY: it exists so that the
reference's own Python (python/qwen35.py, python/delta_kernel.py) can be
executed in a container that has no MLX, to produce golden vectors.  Nothing
in the product imports it.

Semantics follow MLX's documented behaviour where it matters for the GDN path:

* Python scalars are *weak*: ``bf16_array * 0.5`` stays bf16 (numpy alone would
  promote to float32).  bf16 op bf16 -> bf16; bf16 op float32 -> float32.
* Element-wise ops on bf16 compute in float32 and round once to bf16.
* Reductions accumulate in float32 and round to the input dtype.
* ``matmul`` of bf16 operands accumulates in float32 and rounds to bf16.

What is NOT reproduced: MLX's exact reduction order and its transcendental
implementations.  Golden vectors made with this module pin the reference's
*algorithm* (operation order, masks, clips, padding, layouts), not MLX's last
bits.
"""
from __future__ import annotations

import numpy as np
import ml_dtypes

float32 = np.dtype(np.float32)
float16 = np.dtype(np.float16)
bfloat16 = np.dtype(ml_dtypes.bfloat16)
int32 = np.dtype(np.int32)
uint32 = np.dtype(np.uint32)
int64 = np.dtype(np.int64)
bool_ = np.dtype(np.bool_)

_LOW = (bfloat16, float16)


def _is_weak(x):
    return isinstance(x, (bool, int, float)) and not isinstance(x, np.generic)


def _result_dtype(inputs):
    dts = [np.asarray(x).dtype for x in inputs if not _is_weak(x)]
    if not dts:
        return float32
    if all(d == dts[0] for d in dts):
        return dts[0]
    floats = [d for d in dts if d.kind == "f" or d in _LOW]
    if not floats:
        return np.result_type(*dts)
    if any(d == float32 or d == np.float64 for d in floats):
        return float32 if all(d != np.float64 for d in floats) else np.dtype(np.float64)
    if all(d == floats[0] for d in floats):
        return floats[0]
    return float32          # bf16 with f16 -> f32, as MLX promotes


class MxArray(np.ndarray):
    """ndarray with MLX's weak-scalar promotion and low-precision rounding."""

    def __array_ufunc__(self, ufunc, method, *inputs, out=None, **kw):
        target = _result_dtype(inputs)
        raw = []
        for x in inputs:
            if _is_weak(x):
                raw.append(x)
                continue
            a = np.asarray(x).view(np.ndarray)
            if a.dtype in _LOW:
                a = a.astype(np.float32)
            raw.append(a)
        if method == "__call__":
            r = getattr(ufunc, method)(*raw, **kw)
        elif method == "reduce":
            r = ufunc.reduce(*raw, **kw)
        else:
            r = getattr(ufunc, method)(*raw, **kw)
        if isinstance(r, tuple):
            return tuple(_wrap(_cast_like(v, target)) for v in r)
        return _wrap(_cast_like(r, target))

    def item(self, *a):
        return np.asarray(self).view(np.ndarray).item(*a)


def _cast_like(r, target):
    r = np.asarray(r)
    if r.dtype == np.bool_:
        return r
    if target in _LOW or (target == float32 and r.dtype == np.float64):
        return r.astype(target)
    return r


def _wrap(x):
    return np.asarray(x).view(MxArray)


def _raw(x):
    return np.asarray(x).view(np.ndarray)


def _f32(x):
    r = _raw(x)
    return r.astype(np.float32) if r.dtype in _LOW else r


def array(x, dtype=None):
    if isinstance(x, np.ndarray):
        return _wrap(x.astype(dtype) if dtype is not None else x.copy())
    if dtype is None:
        dtype = float32 if isinstance(x, float) or (
            isinstance(x, (list, tuple)) and any(isinstance(v, float) for v in np.ravel(x))) else None
    return _wrap(np.asarray(x, dtype=dtype))


def _shape(s):
    return (s,) if isinstance(s, int) else tuple(s)


def zeros(shape, dtype=float32):
    return _wrap(np.zeros(_shape(shape), dtype=dtype))


def ones(shape, dtype=float32):
    return _wrap(np.ones(_shape(shape), dtype=dtype))


def zeros_like(x):
    return _wrap(np.zeros_like(_raw(x)))


def ones_like(x):
    return _wrap(np.ones_like(_raw(x)))


def eye(n, m=None, k=0, dtype=float32):
    return _wrap(np.eye(n, m, k, dtype=dtype))


def arange(*a, dtype=None):
    r = np.arange(*a)
    if dtype is not None:
        r = r.astype(dtype)
    elif r.dtype == np.int64:
        r = r.astype(np.int32)
    return _wrap(r)


def tril(x, k=0):
    return _wrap(np.tril(_raw(x), k))


def triu(x, k=0):
    return _wrap(np.triu(_raw(x), k))


def _unary(fn):
    def op(x):
        d = _raw(x).dtype
        return _wrap(fn(_f32(x)).astype(d))
    return op


exp = _unary(np.exp)
log = _unary(np.log)
log1p = _unary(np.log1p)
sin = _unary(np.sin)
cos = _unary(np.cos)
abs = _unary(np.abs)
negative = _unary(np.negative)
sqrt = _unary(np.sqrt)
rsqrt = _unary(lambda v: (1.0 / np.sqrt(v)).astype(v.dtype))
sigmoid = _unary(lambda v: (1.0 / (1.0 + np.exp(-v))).astype(v.dtype))


def logaddexp(a, b):
    t = _result_dtype([a, b])
    x, y = _f32(a) if not _is_weak(a) else a, _f32(b) if not _is_weak(b) else b
    return _wrap(np.logaddexp(x, y).astype(t))


def maximum(a, b):
    return _wrap(np.maximum(a, b))


def minimum(a, b):
    return _wrap(np.minimum(a, b))


def clip(x, a_min, a_max):
    d = _raw(x).dtype
    return _wrap(np.clip(_f32(x), a_min, a_max).astype(d))


def where(c, a, b):
    t = _result_dtype([a, b])
    x = a if _is_weak(a) else _f32(a)
    y = b if _is_weak(b) else _f32(b)
    return _wrap(np.where(_raw(c), x, y).astype(t))


def _axis(axis):
    return tuple(axis) if isinstance(axis, list) else axis


def sum(x, axis=None, keepdims=False):
    d = _raw(x).dtype
    return _wrap(np.sum(_f32(x), axis=_axis(axis), keepdims=keepdims).astype(d))


def mean(x, axis=None, keepdims=False):
    d = _raw(x).dtype
    return _wrap(np.mean(_f32(x), axis=_axis(axis), keepdims=keepdims).astype(d))


def max(x, axis=None, keepdims=False):
    return _wrap(np.max(_raw(x), axis=_axis(axis), keepdims=keepdims))


def cumsum(x, axis=None, reverse=False, inclusive=True):
    d = _raw(x).dtype
    v = _f32(x)
    if reverse:
        v = np.flip(v, axis)
    r = np.cumsum(v, axis=axis)
    if not inclusive:
        r = r - v
    if reverse:
        r = np.flip(r, axis)
    return _wrap(r.astype(d))


def matmul(a, b):
    return _wrap(a) @ _wrap(b)


def swapaxes(x, a, b):
    return _wrap(np.swapaxes(_raw(x), a, b))


def transpose(x, axes=None):
    return _wrap(np.transpose(_raw(x), axes))


def reshape(x, shape):
    return _wrap(np.reshape(_raw(x), shape))


def squeeze(x, axis=None):
    return _wrap(np.squeeze(_raw(x), axis))


def expand_dims(x, axis):
    return _wrap(np.expand_dims(_raw(x), axis))


def broadcast_to(x, shape):
    return _wrap(np.broadcast_to(_raw(x), shape))


def concatenate(arrays, axis=0):
    return _wrap(np.concatenate([_raw(a) for a in arrays], axis=axis))


def stack(arrays, axis=0):
    return _wrap(np.stack([_raw(a) for a in arrays], axis=axis))


def repeat(x, repeats, axis=None):
    return _wrap(np.repeat(_raw(x), repeats, axis=axis))


def take(x, idx, axis=None):
    return _wrap(np.take(_raw(x), _raw(idx), axis=axis))


def contiguous(x):
    return _wrap(np.ascontiguousarray(_raw(x)).copy())


def eval(*args):
    return None


def compile(fn=None, shapeless=False, **kw):
    if fn is None:
        return lambda f: f
    return fn


class _Finfo:
    def __init__(self, d):
        f = np.finfo(np.float32 if d in _LOW else d)
        self.max = float(f.max)
        self.min = float(f.min)


def finfo(d):
    return _Finfo(np.dtype(d))


class _Device:
    def __init__(self, name):
        self.name = name

    def __eq__(self, other):
        return isinstance(other, _Device) and other.name == self.name

    def __hash__(self):
        return hash(self.name)


gpu = _Device("gpu")
cpu = _Device("cpu")


def default_device():
    return cpu


class metal:  # noqa: N801 - mirrors the mlx.core.metal namespace
    @staticmethod
    def is_available():
        return False


class fast:  # noqa: N801 - mirrors the mlx.core.fast namespace
    @staticmethod
    def rms_norm(x, weight, eps):
        """x * rsqrt(mean(x^2, -1) + eps) * weight, computed in float32 and
        returned in x's dtype (MLX's documented definition)."""
        d = _raw(x).dtype
        v = _f32(x)
        r = v * (1.0 / np.sqrt(np.mean(v * v, axis=-1, keepdims=True) + np.float32(eps)))
        if weight is not None:
            r = r * _f32(weight)
        return _wrap(r.astype(d))

    @staticmethod
    def metal_kernel(*a, **kw):
        raise RuntimeError("no Metal in the numpy MLX stand-in")
