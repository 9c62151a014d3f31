"""GDN-2 fused backward on B200 (mirrors the reference module gdn2_bwd.py).

The reference splits the backward into B1 (state), B2 (dAqk/dv), B3 (WY),
B4 (scores) and B5 (reverse cumsum) (gdn2_bwd.py:32, 45, 99, 213, 342).  Here
they run as one reverse state kernel (B1 with B2's dv) and three intra-chunk
kernels (B2's dAqk + B3, B3's WY half, B4 + B5 + assembly) inside
libgdn2.so; ``gdn2_backward`` is the single entry point.
"""
from __future__ import annotations

import torch

from . import _lib
from . import gdn2_fwd as _fwd


def gdn2_backward(q, k, v, w, b, g, scale, h0, dout, dh_final, workspace=None):
    """Cotangents (dq, dk, dv, dw, db, dg, dh0) of (o, h_final) w.r.t. the
    inputs, as _gdn2_core_bwd returns them (gdn2_pipeline.py:70-137): final
    +-1e4 sanitiser, each gradient cast to its input's dtype.

    ``workspace`` may be the buffer a previous forward filled with residuals
    (``gdn2_pallas_forward_trainable`` does this) to skip the recompute of
    the forward; without it the forward is recomputed as in the reference.
    """
    p = _fwd._Prepared(q, k, v, w, b, g, scale, h0)
    dev = p.dev
    do = torch.as_tensor(dout).to(device=dev, dtype=torch.float32, non_blocking=True).contiguous()
    if tuple(do.shape) != (p.B, p.T_user, p.H, p.D):
        raise _fwd.Gdn2ShapeError(f"dout must be {(p.B, p.T_user, p.H, p.D)}")
    do = p.pad(do)
    if dh_final is None:
        dhf = torch.zeros((p.B, p.H, p.D, p.D), dtype=torch.float32, device=dev)
    else:
        dhf = torch.as_tensor(dh_final).to(device=dev, dtype=torch.float32,
                                           non_blocking=True).contiguous()
        if tuple(dhf.shape) != (p.B, p.H, p.D, p.D):
            raise _fwd.Gdn2ShapeError(f"dh_final must be {(p.B, p.H, p.D, p.D)}")
    residuals_valid = workspace is not None
    ws = workspace if residuals_valid else p.workspace(True)
    grads = [torch.empty((p.B, p.T, p.H, p.D), dtype=p.dtype, device=dev) for _ in range(6)]
    dh0 = torch.empty((p.B, p.H, p.D, p.D), dtype=torch.float32, device=dev)
    dq, dk, dv, dw, db, dg = grads
    rc = _lib.load().gdn2_bwd(
        p.code, *p.ptrs(), p.h0.data_ptr() if p.h0 is not None else None, do.data_ptr(),
        dhf.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dw.data_ptr(),
        db.data_ptr(), dg.data_ptr(), dh0.data_ptr(), ws.data_ptr(), ws.numel(),
        int(residuals_valid), p.B, p.T, p.H, p.D, p.C, p.bc, p.scale, p.clip, p.stream)
    _lib.check(rc, "gdn2_bwd")
    _lib.check_status(ws, p.stream, "gdn2_bwd", synced=p.on_host)
    out = [p.unpad(t) for t in (dq, dk, dv, dw, db, dg)]
    order = (0, 1, 2, 3, 4, 5)  # q k v w b g
    out = [t.to(p.in_dtypes[i]) for t, i in zip(out, order)]
    dh0 = dh0.to(p.h0_dtype)
    if p.on_host:
        out = [t.cpu() for t in out]
        dh0 = dh0.cpu()
    return (*out, dh0)
