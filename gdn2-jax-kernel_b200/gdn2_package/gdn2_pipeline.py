"""Trainable GDN-2 (mirrors the reference module gdn2_pipeline.py).

``gdn2_pallas_forward_trainable(q,k,v,w,b,g,scale,h0=None)`` returns
``(out, h_final)`` and is differentiable w.r.t. q, k, v, w, b, g and h0;
``scale`` is not (the reference's custom_vjp with nondiff_argnums=(6,),
gdn2_pipeline.py:59-61, 143-159).  In PyTorch the custom VJP is a
``torch.autograd.Function``; its backward returns the reference's cotangents
(dq, dk, dv, dw, db, dg, dh0) (gdn2_pipeline.py:137).

By default the forward keeps its per-chunk state in the workspace so the
backward skips the forward recompute; ``recompute=True`` instead saves only
the inputs, exactly like the reference (gdn2_pipeline.py:64-67).
"""
from __future__ import annotations

import torch

from . import gdn2_bwd as _bwd
from . import gdn2_fwd as _fwd

_FINAL_CLIP = 1e4  # gdn2_pipeline.py:34


def _gdn2_core_fwd(q, k, v, w, b, g, scale, h0, keep_residuals=True):
    """Forward rule: returns ((out, h_final), residuals) (gdn2_pipeline.py:64-67)."""
    if _fwd._head_dim(q) in _fwd._STAGE_D:   # stage kernels; the backward recomputes
        o, h_final = _fwd.gdn2_pallas_forward(q, k, v, w, b, g, scale, h0)
        return (o, h_final), (q, k, v, w, b, g, h0, None)
    p = _fwd._Prepared(q, k, v, w, b, g, scale, h0)
    o, h_final, ws = _fwd._run_forward(p, save_residuals=keep_residuals)
    residuals = (q, k, v, w, b, g, h0, ws if keep_residuals else None)
    return (o, h_final), residuals


def _gdn2_core_bwd(scale, residuals, cotangents):
    """Backward rule: returns (dq, dk, dv, dw, db, dg, dh0) (gdn2_pipeline.py:70-137)."""
    q, k, v, w, b, g, h0 = residuals[:7]
    ws = residuals[7] if len(residuals) > 7 else None
    do, dh_final = cotangents
    return _bwd.gdn2_backward(q, k, v, w, b, g, scale, h0, do, dh_final, workspace=ws)


class _Gdn2Core(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, w, b, g, h0, scale, recompute):
        (o, h_final), res = _gdn2_core_fwd(q, k, v, w, b, g, scale, h0,
                                           keep_residuals=not recompute)
        ctx.scale = scale
        ctx.ws = res[7]
        ctx.save_for_backward(q, k, v, w, b, g, h0)
        return o, h_final

    @staticmethod
    def backward(ctx, do, dh_final):
        q, k, v, w, b, g, h0 = ctx.saved_tensors
        if do is None:
            do = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        grads = _gdn2_core_bwd(ctx.scale, (q, k, v, w, b, g, h0, ctx.ws), (do, dh_final))
        ctx.ws = None
        dq, dk, dv, dw, db, dg, dh0 = grads
        return dq, dk, dv, dw, db, dg, dh0, None, None


def gdn2_pallas_forward_trainable(q, k, v, w, b, g, scale, h0=None, recompute=False):
    """Trainable Gated DeltaNet-2 forward with the fused backward.

    Args: q, k, v, w, b, g (batch, seq_len, heads, d_head) CUDA tensors;
    scale a Python float; h0 (batch, heads, d_head, d_head), zero if None.
    Returns out (batch, seq_len, heads, d_head) and h_final
    (batch, heads, d_head, d_head), both float32.
    """
    B, T, H, D = q.shape
    if h0 is None:
        h0 = torch.zeros((B, H, D, D), dtype=torch.float32, device=q.device)
    return _Gdn2Core.apply(q, k, v, w, b, g, h0, float(scale), bool(recompute))
