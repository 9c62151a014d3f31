"""ctypes wrapper of oracle/gdn2_cpu.cpp, the fp32 C++/OpenMP restatement of
the reference algorithm used as the timed CPU baseline (test and benchmark
infrastructure; the product path never loads it).

    python oracle/gdn2_cpu.py          # builds oracle/_build/libgdn2cpu.so
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "gdn2_cpu.cpp")
LIB = os.path.join(HERE, "_build", "libgdn2cpu.so")
_lib = None


def build(force=False):
    """Compile the restatement with g++ -O3 -fopenmp (no-op when up to date)."""
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    tmp = LIB + ".tmp"
    subprocess.check_call(["g++", "-O3", "-march=x86-64-v3", "-fopenmp", "-shared", "-fPIC", SRC,
                           "-o", tmp])
    os.replace(tmp, LIB)
    return LIB


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        _lib = ctypes.CDLL(LIB)
        _lib.gdn2_cpu_fwd_bwd.restype = ctypes.c_int
    return _lib


def fwd_bwd(inp, BT, BC, clip, threads=0, backward=True):
    """Run the restatement on a dict of (B, T, H, D) arrays (make_inputs
    layout).  Returns (o, h_final, (dq, dk, dv, dw, db, dg, dh0) or None)."""
    f = lambda a: np.ascontiguousarray(a, np.float32)
    xs = [f(inp[n]) for n in ("q", "k", "v", "w", "b", "g")]
    B, T, H, D = xs[0].shape
    h0 = f(inp["h0"]) if inp.get("h0") is not None else None
    do = f(inp["dout"]) if backward else None
    dhf = f(inp["dh_final"]) if backward else None
    o = np.zeros((B, T, H, D), np.float32)
    hf = np.zeros((B, H, D, D), np.float32)
    grads = [np.zeros((B, T, H, D), np.float32) for _ in range(6)] if backward else []
    dh0 = np.zeros((B, H, D, D), np.float32) if backward else None
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p) if a is not None else None
    gp = [p(a) for a in grads] if backward else [None] * 6
    rc = load().gdn2_cpu_fwd_bwd(*[p(a) for a in xs], p(h0), p(do), p(dhf), p(o), p(hf), *gp,
                                 p(dh0), B, T, H, D, BT, BC, ctypes.c_float(inp["scale"]),
                                 ctypes.c_float(clip), int(threads))
    if rc:
        raise ValueError("gdn2_cpu_fwd_bwd: invalid sizes")
    return o, hf, ((*grads, dh0) if backward else None)


if __name__ == "__main__":
    print(build(force=True))
