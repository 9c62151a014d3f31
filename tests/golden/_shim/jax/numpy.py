"""numpy-backed subset of ``jax.numpy`` (see the package docstring)."""
import os
import numpy as _np

float32 = _np.dtype(os.environ.get("GDN2_SHIM_DTYPE", "float64"))
float64 = _np.dtype("float64")
ndarray = _np.ndarray


def _f(x):
    return _np.asarray(x)


def nan_to_num(x, nan=0.0, posinf=None, neginf=None):
    return _np.nan_to_num(_f(x), nan=nan, posinf=posinf, neginf=neginf)


def clip(x, lo, hi):
    return _np.clip(_f(x), lo, hi)


def dot(a, b, precision=None):
    return _np.dot(_f(a), _f(b))


def einsum(spec, *ops, precision=None):
    return _np.einsum(spec, *[_f(o) for o in ops])


def arange(n):
    return _np.arange(n)


def zeros(shape, dtype=None):
    return _np.zeros(shape, dtype=float32 if dtype is None else dtype)


def ones(shape, dtype=None):
    return _np.ones(shape, dtype=float32 if dtype is None else dtype)


def zeros_like(x):
    return _np.zeros_like(_f(x))


def concatenate(xs, axis=0):
    return _np.concatenate([_f(x) for x in xs], axis=axis)


def moveaxis(x, src, dst):
    return _np.moveaxis(_f(x), src, dst)


exp = _np.exp
sum = _np.sum
abs = _np.abs
max = _np.max
all = _np.all
where = _np.where
isfinite = _np.isfinite
logical_not = _np.logical_not
asarray = _np.asarray
