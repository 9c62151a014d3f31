"""Generate golden vectors by executing the reference GDN-2 source itself.

The reference (Akseleu-J/gdn2-jax-kernel: gdn2_fwd.py, gdn2_bwd.py,
gdn2_pipeline.py) is JAX/Pallas code and JAX is not installable here, so the
reference modules are imported unmodified on top of ``_shim/jax`` — a numpy
interpreter for the JAX calls they make (``pallas_call`` grids run eagerly over
numpy views, ``lax.scan``/``fori_loop`` run as Python loops).  With
``GDN2_SHIM_DTYPE=float64`` the reference algorithm runs without float32
rounding, which pins the float64 oracle under ``oracle/``.

Harness-level adjustments, each needed for the reference to run at all:
  * module constants BT/BC/N_SUB/CLIP are set in every module that copied them
    at import (gdn2_fwd.py:29-33, gdn2_bwd.py:23, gdn2_pipeline.py:14-15);
  * ``gdn2_inter_chunk_combine_with_state`` returns h_pre_all / v_new_all
    chunk-major (gdn2_fwd.py:393-397) while B1/B2/B3 index them batch-major
    (gdn2_bwd.py:104, 224); the wrapper below moves the chunk axis to axis 2
    before the pipeline sees them (the intended layout);
  * only N_SUB == 2 and D == 128 are used, the cases the reference computes
    correctly (gdn2_fwd.py:145, 228-243).

Run in this repository's container (needs the reference checkout):
    python tests/golden/make_golden.py /path/to/reference
Writes ``tests/golden/*.npz``.  The GPU box never runs this script.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_reference(ref_dir, BT, BC, clip):
    os.environ.setdefault("GDN2_SHIM_DTYPE", "float64")
    sys.path.insert(0, os.path.join(HERE, "_shim"))
    sys.path.insert(0, ref_dir)
    for m in ("gdn2_fwd", "gdn2_bwd", "gdn2_pipeline"):
        sys.modules.pop(m, None)
    import gdn2_fwd as fwd  # noqa: E402
    import gdn2_bwd as bwd  # noqa: E402
    import gdn2_pipeline as pipe  # noqa: E402

    for mod in (fwd, bwd):
        mod.BT, mod.BC, mod.N_SUB, mod.CLIP = BT, BC, BT // BC, clip
    pipe.BT = BT

    orig = fwd.gdn2_inter_chunk_combine_with_state

    def with_state_batch_major(*a, **kw):
        o, h_final, h_pre_all, v_new_all = orig(*a, **kw)
        return o, h_final, np.moveaxis(h_pre_all, 0, 2), np.moveaxis(v_new_all, 0, 2)

    pipe.gdn2_inter_chunk_combine_with_state = with_state_batch_major
    return fwd, bwd, pipe


def run_case(ref_dir, name, B, T, H, D, BT, BC, clip, seed, h0_std, ones=False, dscale=1.0):
    sys.path.insert(0, os.path.join(HERE, "..", "..", "gdn2-jax-kernel_b200"))
    from gdn2_package.synthetic import make_inputs

    fwd, bwd, pipe = _load_reference(ref_dir, BT, BC, clip)
    inp = make_inputs(B, T, H, D, seed=seed, h0_std=h0_std)
    if ones:
        for n in ("q", "k", "v", "w", "b", "g"):
            inp[n] = np.ones_like(inp[n])
        inp["scale"] = 0.1
    # upstream gradients scaled so that the clip acts inside the backward chain
    inp["dout"] = (inp["dout"] * dscale).astype(np.float32)
    inp["dh_final"] = (inp["dh_final"] * dscale).astype(np.float32)
    f64 = lambda a: np.asarray(a, dtype=np.float64)
    q, k, v, w, b, g = (f64(inp[n]) for n in ("q", "k", "v", "w", "b", "g"))
    h0 = f64(inp["h0"]) if "h0" in inp else np.zeros((B, H, D, D))
    scale = inp["scale"]

    (o, h_final), res = pipe._gdn2_core_fwd(q, k, v, w, b, g, scale, h0)
    dq, dk, dv, dw, db, dg, dh0 = pipe._gdn2_core_bwd(
        scale, res, (f64(inp["dout"]), f64(inp["dh_final"])))
    o2, h2 = fwd.gdn2_pallas_forward(q, k, v, w, b, g, scale, h0=h0)
    assert np.array_equal(o, o2) and np.array_equal(h_final, h2)

    out = dict(q=q, k=k, v=v, w=w, b=b, g=g, h0=h0, dout=inp["dout"],
               dh_final=inp["dh_final"], o=o, h_final=h_final, dq=dq, dk=dk,
               dv=dv, dw=dw, db=db, dg=dg, dh0=dh0)
    out = {n: np.asarray(a, dtype=np.float32) for n, a in out.items()}
    meta = np.array([B, T, H, D, BT, BC], dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), meta=meta,
                        clip=np.float64(clip), scale=np.float64(scale), **out)
    print(name, "o", float(np.abs(o).max()), "h", float(np.abs(h_final).max()),
          "dq", float(np.abs(dq).max()), "dg", float(np.abs(dg).max()))


CASES = [
    # name, B, T, H, D, BT, BC, clip, seed, h0_std, ones, dout scale
    ("ref_bt64_bc32", 1, 128, 1, 128, 64, 32, 1e4, 1, 0.1, False, 1.0),
    ("ref_bt128_bc64", 1, 256, 1, 128, 128, 64, 1e3, 2, None, False, 1.0),
    ("ref_ones_bt64_bc32", 1, 128, 1, 128, 64, 32, 1e4, 3, None, True, 1.0),
    # CLIP = 20 with dout, dh_final x 30: dv_new = san(dv_partial + kg dh)
    # clips inside the backward state chain (gdn2_bwd.py:66-68), h and dh do not
    ("ref_clip_bt128_bc64", 1, 512, 1, 128, 128, 64, 20.0, 4, 0.1, False, 30.0),
]

if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GDN2_REFERENCE_DIR")
    if not ref:
        sys.exit("usage: make_golden.py <reference checkout>")
    only = sys.argv[2:]   # optional case names
    for c in CASES:
        if not only or c[0] in only:
            run_case(ref, *c[:-2], ones=c[-2], dscale=c[-1])
