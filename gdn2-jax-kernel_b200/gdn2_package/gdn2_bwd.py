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

_FINAL_CLIP = 1e4  # gdn2_pipeline.py:34


def gdn2_backward(q, k, v, w, b, g, scale, h0, dout, dh_final, workspace=None, _prep_done=False):
    """Cotangents (dq, dk, dv, dw, db, dg, dh0) of (o, h_final) w.r.t. the
    inputs, as _gdn2_core_bwd returns them (gdn2_pipeline.py:70-137): final
    +-1e4 sanitiser, each gradient cast to its input's dtype.

    ``workspace`` may be the buffer a previous forward filled with residuals
    (``gdn2_pallas_forward_trainable`` does this) to skip the recompute of
    the forward; without it the forward is recomputed as in the reference.  ``_prep_done`` (internal:
    sequence_parallel / segmented): a gdn2_sp_segment op 2 with this same
    dout already formed the per-chunk backward terms in ``workspace``.
    """
    if _fwd._head_dim(q) in _fwd._STAGE_D:
        return _stage_backward(q, k, v, w, b, g, scale, h0, dout, dh_final)
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
        (2 if _prep_done else 1) if residuals_valid else 0, p.B, p.T, p.H, p.D, p.C, p.bc,
        p.scale, p.clip, p.stream)
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


# ---------- the reference's stage functions (B1-B5, gdn2_bwd.py:32-375) ----------
# Separate entry points on the reference's chunked layouts (one CUDA kernel
# of libgdn2.so each, gdn2_stage_*); gdn2_backward above does not use them.

def _dev_of(t):
    t = torch.as_tensor(t)
    return t.device if t.device.type == "cuda" else torch.device("cuda", torch.cuda.current_device())


def reverse_cumsum_bwd(dgc, chunk_size):
    """B5: dg_raw[i] = san(sum_{j >= i} dgc[j]) within each chunk of
    ``chunk_size`` rows (gdn2_bwd.py:32-41); dgc is (..., chunk_size, D)."""
    dev = _dev_of(dgc)
    x = _fwd._f32(dgc, dev)
    C, D = x.shape[-2], x.shape[-1]
    if C != int(chunk_size):
        raise _fwd.Gdn2ShapeError(f"dgc's chunk axis is {C}, chunk_size={chunk_size}")
    out = torch.empty_like(x)
    rc = _lib.load().gdn2_stage_revcumsum(x.data_ptr(), out.data_ptr(), x.numel() // (C * D), C, D,
                                          float(_fwd.CLIP), _fwd._stream(dev))
    _lib.check(rc, "reverse_cumsum_bwd")
    return out


def gdn2_dhu_backward(do, dv_partial, w_pseudo, qg, kg, gc_last, scale, dht=None):
    """B1: dh_all (B, H, nc, D, D), dh0 (B, H, D, D), dv_all (B, H, nc, BT, D)
    (gdn2_bwd.py:45-80); do is chunked (B, H, nc, BT, D)."""
    dev = _dev_of(qg)
    xs = [_fwd._f32(t, dev) for t in (do, dv_partial, w_pseudo, qg, kg, gc_last)]
    B, H, nc, bt, D = xs[3].shape
    dht = None if dht is None else _fwd._f32(dht, dev)
    dh_all = torch.empty((B, H, nc, D, D), dtype=torch.float32, device=dev)
    dh0 = torch.empty((B, H, D, D), dtype=torch.float32, device=dev)
    dv_all = torch.empty((B, H, nc, bt, D), dtype=torch.float32, device=dev)
    rc = _lib.load().gdn2_stage_dhu(*[t.data_ptr() for t in xs],
                                    dht.data_ptr() if dht is not None else None,
                                    dh_all.data_ptr(), dh0.data_ptr(), dv_all.data_ptr(), B, H, nc,
                                    bt, D, float(scale), float(_fwd.CLIP), _fwd._stream(dev))
    _lib.check(rc, "gdn2_dhu_backward")
    return dh_all, dh0, dv_all


def dav_backward_pallas(Aqk, v_new, do):
    """B2: dAqk = san((do v_new^T) * causal), dv_new = san(Aqk^T do)
    (gdn2_bwd.py:84-122); all (B, H, nc, ., .)."""
    dev = _dev_of(v_new)
    aqk, vn, d = (_fwd._f32(t, dev) for t in (Aqk, v_new, do))
    B, H, nc, bt, D = vn.shape
    daqk = torch.empty_like(aqk)
    dv = torch.empty_like(vn)
    rc = _lib.load().gdn2_stage_dav(aqk.data_ptr(), vn.data_ptr(), d.data_ptr(), daqk.data_ptr(),
                                    dv.data_ptr(), B * H * nc, bt, D, float(_fwd.CLIP),
                                    _fwd._stream(dev))
    _lib.check(rc, "dav_backward_pallas")
    return daqk, dv


def wy_dqkg_backward_pallas(q, k, b, w, v, gc, A, Akk, h_pre_all, v_new_all, do, dv, dh_next_all,
                            scale):
    """B3: dict of dq, dk, db, dw, dv_raw, dgc (B, H, nc, BT, D) and dAkk
    (B, H, nc, BT, BT) (gdn2_bwd.py:126-244).  Every argument is chunked
    batch-major; Akk is not read (as in the reference)."""
    del Akk
    dev = _dev_of(q)
    xs = [_fwd._f32(t, dev) for t in (q, k, b, w, v, gc, A, h_pre_all, v_new_all, do, dv,
                                      dh_next_all)]
    B, H, nc, bt, D = xs[0].shape
    outs = [torch.empty((B, H, nc, bt, D), dtype=torch.float32, device=dev) for _ in range(6)]
    dakk = torch.empty((B, H, nc, bt, bt), dtype=torch.float32, device=dev)
    scratch = torch.empty_like(dakk)
    rc = _lib.load().gdn2_stage_wy_dqkg(*[t.data_ptr() for t in xs],
                                        *[t.data_ptr() for t in outs], dakk.data_ptr(),
                                        scratch.data_ptr(), B * H * nc, bt, D, float(scale),
                                        float(_fwd.CLIP), _fwd._stream(dev))
    _lib.check(rc, "wy_dqkg_backward_pallas")
    dq, dk, db, dw, dv_raw, dgc = outs
    return dict(dq=dq, dk=dk, db=db, dw=dw, dv_raw=dv_raw, dgc=dgc, dAkk=dakk)


def intra_backward_pallas(dAqk, dAkk, q, k, b, g, scale):
    """B4: dq, dk, db, dgc (B, H, nc, BT, D) from the score gradients, in the
    reference's sub-block pair order with its clipped accumulation
    (gdn2_bwd.py:248-375); q, k, b, g are (B, L, H, D)."""
    B, L, H, D, bt = _fwd._check_seq(torch.as_tensor(q))
    (q, k, b, g), code, dev = _fwd._stage_in((q, k, b, g))
    tr = lambda t: _fwd._f32(t, dev).transpose(-1, -2).contiguous()
    daqkT, dakkT = tr(dAqk), tr(dAkk)
    nc = L // bt
    outs = [torch.empty((B, H, nc, bt, D), dtype=torch.float32, device=dev) for _ in range(4)]
    zeros = torch.zeros((bt, D), dtype=torch.float32, device=dev)
    rc = _lib.load().gdn2_stage_intra_bwd(code, daqkT.data_ptr(), dakkT.data_ptr(), q.data_ptr(),
                                          k.data_ptr(), b.data_ptr(), g.data_ptr(),
                                          zeros.data_ptr(), *[t.data_ptr() for t in outs], B, L, H,
                                          D, bt, int(_fwd.BC), float(scale), float(_fwd.CLIP),
                                          _fwd._stream(dev))
    _lib.check(rc, "intra_backward_pallas")
    return tuple(outs)


def _stage_backward(q, k, v, w, b, g, scale, h0, dout, dh_final):
    """Backward of a head dim the fused kernels do not cover (D = 256): the
    reference's _gdn2_core_bwd (gdn2_pipeline.py:70-137) composed of the
    stage kernels, with the final +-1e4 sanitiser and the input dtypes."""
    q_t = torch.as_tensor(q)
    B, L, H, D, bt = _fwd._check_seq(q_t)
    nc = L // bt
    (qd, kd, vd, wd, bd, gd), _, dev = _fwd._stage_in((q, k, v, w, b, g))
    f32 = lambda t: None if t is None else _fwd._f32(t, dev)
    h0d, do, dhf = f32(h0), f32(dout), f32(dh_final)
    if tuple(do.shape) != (B, L, H, D):
        raise _fwd.Gdn2ShapeError(f"dout must be {(B, L, H, D)}")
    if dhf is None:
        dhf = torch.zeros((B, H, D, D), dtype=torch.float32, device=dev)
    Aqk, Akk = _fwd.build_chunk_scores_pallas(qd, kd, bd, gd, scale)
    A = _fwd.wy_solve_pallas(Akk)
    wp, u, kg, qg, gcl = _fwd.recompute_wy_pallas(qd, kd, vd, wd, bd, gd, A)
    _, _, hpre, vall = _fwd.gdn2_inter_chunk_combine_with_state(Aqk, wp, u, kg, qg, gcl, scale, h0d)
    hpre, vall = hpre.permute(1, 2, 0, 3, 4), vall.permute(1, 2, 0, 3, 4)
    ch = lambda t: t.float().reshape(B, nc, bt, H, D).permute(0, 3, 1, 2, 4).contiguous()
    # gc = in-chunk cumsum of g (gdn2_pipeline.py:94-96)
    gc = torch.cumsum(ch(gd).double(), dim=-2).float()
    dAqk, dvp = dav_backward_pallas(Aqk, vall, ch(do))
    dh_all, dh0, dv_all = gdn2_dhu_backward(ch(do), dvp, wp, qg, kg, gcl, scale, dht=dhf)
    dh_next = torch.cat([dh_all[:, :, 1:], dhf[:, :, None]], dim=2)   # gdn2_pipeline.py:52-56
    b3 = wy_dqkg_backward_pallas(ch(qd), ch(kd), ch(bd), ch(wd), ch(vd), gc, A, Akk, hpre, vall,
                                 ch(do), dv_all, dh_next, scale)
    dq4, dk4, db4, dgc4 = intra_backward_pallas(dAqk, b3["dAkk"], qd, kd, bd, gd, scale)
    dg = reverse_cumsum_bwd(b3["dgc"] + dgc4, bt)
    unch = lambda t: t.permute(0, 2, 3, 1, 4).reshape(B, L, H, D)
    fin = lambda t: torch.nan_to_num(t.clamp(-_FINAL_CLIP, _FINAL_CLIP), nan=0.0,
                                     posinf=_FINAL_CLIP, neginf=-_FINAL_CLIP)
    grads = [fin(unch(t)) for t in (b3["dq"] + dq4, b3["dk"] + dk4, b3["dv_raw"], b3["dw"],
                                    b3["db"] + db4, dg)]
    ins = [torch.as_tensor(t) for t in (q, k, v, w, b, g)]
    grads = [t.to(x.dtype) for t, x in zip(grads, ins)]
    dh0 = fin(dh0)
    if h0 is not None:
        dh0 = dh0.to(torch.as_tensor(h0).dtype)
    if ins[0].device.type != "cuda":
        grads = [t.cpu() for t in grads]
        dh0 = dh0.cpu()
    return (*grads, dh0)
