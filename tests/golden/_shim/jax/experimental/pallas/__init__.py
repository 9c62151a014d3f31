"""Eager numpy interpreter for ``pl.pallas_call`` with ``BlockSpec`` grids.

Each grid point runs the kernel body once; every ref is a numpy view of the
block that the spec's index map selects (block index × block shape), so reads
copy values and writes land in the output buffer, as in Pallas interpret mode.
"""
import itertools
import numpy as _np

from . import tpu  # noqa: F401


class BlockSpec:
    def __init__(self, block_shape, index_map):
        self.block_shape = tuple(block_shape)
        self.index_map = index_map


class _Ref:
    def __init__(self, view):
        self._v = view

    def __getitem__(self, idx):
        return _np.array(self._v[idx])

    def __setitem__(self, idx, val):
        self._v[idx] = val

    @property
    def shape(self):
        return self._v.shape


def _block(arr, spec, gidx):
    bidx = spec.index_map(*gidx)
    sl = tuple(slice(int(b) * s, (int(b) + 1) * s) for b, s in zip(bidx, spec.block_shape))
    return arr[sl]


def pallas_call(kernel, grid, in_specs, out_specs, out_shape, compiler_params=None, **_):
    single = not isinstance(out_shape, (list, tuple))
    outs_meta = [out_shape] if single else list(out_shape)
    ospecs = [out_specs] if single else list(out_specs)

    def run(*inputs):
        ins = [_np.asarray(x) for x in inputs]
        outs = [_np.zeros(m.shape, dtype=m.dtype) for m in outs_meta]
        for gidx in itertools.product(*[range(n) for n in grid]):
            refs = [_Ref(_block(a, s, gidx)) for a, s in zip(ins, in_specs)]
            refs += [_Ref(_block(o, s, gidx)) for o, s in zip(outs, ospecs)]
            kernel(*refs)
        return outs[0] if single else outs

    return run
