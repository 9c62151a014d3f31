"""Minimal numpy-backed stand-in for the parts of the JAX API that the
reference GDN-2 modules use, so that their own source can be executed on a
CPU without jaxlib.  Test infrastructure only: used by ``make_golden.py`` to
produce golden vectors, never by the library.

Semantics follow the published JAX documentation of each function (eager,
no tracing).  The working float type is chosen by the environment variable
``GDN2_SHIM_DTYPE`` (``float64`` by default): the reference casts everything
to ``jnp.float32``, which this shim maps to that type, so a float64 run
executes the reference algorithm without float32 rounding.
"""
import os
import numpy as _np

from . import numpy  # noqa: F401
from . import lax  # noqa: F401
from . import debug  # noqa: F401
from . import experimental  # noqa: F401

float32 = numpy.float32


class ShapeDtypeStruct:
    def __init__(self, shape, dtype):
        self.shape = tuple(shape)
        self.dtype = dtype


class custom_vjp:
    """Eager custom_vjp: calling the object evaluates the primal function.
    ``defvjp`` stores the rules so a caller can invoke them directly."""

    def __init__(self, fun, nondiff_argnums=()):
        self.fun = fun
        self.nondiff_argnums = nondiff_argnums
        self.fwd = None
        self.bwd = None

    def defvjp(self, fwd, bwd):
        self.fwd, self.bwd = fwd, bwd

    def __call__(self, *args):
        return self.fun(*args)


def devices(kind=None):
    raise RuntimeError("numpy shim: no accelerator devices")
