"""numpy-backed subset of ``jax.lax`` (see the package docstring)."""
import numpy as _np


class Precision:
    DEFAULT = "default"
    HIGH = "high"
    HIGHEST = "highest"


def fori_loop(lo, hi, body, init):
    val = init
    for i in range(lo, hi):
        val = body(i, val)
    return val


def cond(pred, true_fun, false_fun, *operands):
    return true_fun(*operands) if bool(pred) else false_fun(*operands)


def _stack(items):
    first = items[0]
    if first is None:
        return None
    if isinstance(first, tuple):
        return tuple(_stack([it[i] for it in items]) for i in range(len(first)))
    return _np.stack([_np.asarray(it) for it in items], axis=0)


def scan(f, init, xs, reverse=False):
    """Eager ``lax.scan`` over the leading axis of a tuple/array of inputs."""
    if isinstance(xs, tuple):
        n = xs[0].shape[0]
        get = lambda i: tuple(x[i] for x in xs)
    else:
        n = xs.shape[0]
        get = lambda i: xs[i]
    order = range(n - 1, -1, -1) if reverse else range(n)
    carry = init
    ys = [None] * n
    for i in order:
        carry, y = f(carry, get(i))
        ys[i] = y
    return carry, _stack(ys)
