"""Chunk-parallel recurrence on one GPU, for few long sequences.

The inter-chunk scan walks the chunks of one (batch, head) in order, one CTA
per (batch, head).  With few of them (config 3: B1 H8, T = 131072, 1024
chunks) most of the 148 SMs idle through the scans.  This mode cuts every
sequence into S equal time segments and runs them as S * B sequences of
length T / S (a reshape: segment s of batch b is batch b * S + s), which
multiplies the scan's parallelism by S and divides its chain by S.  The
segments are then joined exactly as the sequence-parallel ranks are
(sequence_parallel.py): each segment's affine map h_end = P h_start + c
(gdn2_sp_segment op 0), the start states composed in float64, one rescan
(op 1); the backward composes the incoming state gradients the other way
(op 2) and runs the ordinary backward of every segment from its true start
state and incoming gradient.  The reference scans serially
(gdn2_fwd.py:362, gdn2_bwd.py:77); the composition equals it while no state
sanitiser acts on the chain (the clip of h and dh to +-CLIP and of dv_new,
gdn2_fwd.py:358, gdn2_bwd.py:68-73).  The kernels flag every such event in
the workspace status; a flagged forward or backward is rerun here on the
serial path, so the result is the reference's function either way.
"""
from __future__ import annotations

import torch

from . import _lib
from . import gdn2_bwd as _bwd
from . import gdn2_fwd as _fwd
from . import sequence_parallel as _sp

_FINAL_CLIP = 1e4        # gdn2_pipeline.py:34
MIN_SEGMENT_CHUNKS = 16  # shorter segments spend more on the joins than they save


def plan_segments(B, T, H, C, sms):
    """Segments per sequence: 1 (no split) unless the (batch, head) scans
    fill at most an eighth of the SMs; then the largest power of two S >= 2
    with B * H * S <= sms CTAs and segments of at least MIN_SEGMENT_CHUNKS
    whole chunks.  (Measured on B200: config 3, 8 scans, 34.4 -> 24.3 ms per
    fwd+bwd step with S = 16; config 1, 48 scans, 8.8 -> 10.7 ms with S = 2:
    the joins cost passes of per-chunk work that outweigh the shorter chains
    once the scans already occupy a third of the SMs.)"""
    S = 1
    if B * H * 8 > sms:
        return S
    while (B * H * S * 2 <= sms and T % (S * 2 * C) == 0
           and T // (S * 2 * C) >= MIN_SEGMENT_CHUNKS):
        S *= 2
    return S


def _split(x, S):
    B, T, H, D = x.shape
    return x.reshape(B * S, T // S, H, D)


class SegmentedState:
    """What the backward needs: the segment run's state and the maps."""

    def __init__(self, st, S, B, maps):
        self.st, self.S, self.B, self.maps = st, S, B, maps


def _compose_forward(P, c, h0, S):
    """h_start of every segment (B * S, H, D, D) and h_final, in float64."""
    B = P.shape[0] // S
    P = P.view(B, S, *P.shape[1:]).double()
    c = c.view(B, S, *c.shape[1:]).double()
    h = h0.double()
    starts = []
    for s in range(S):
        starts.append(h)
        h = P[:, s] @ h + c[:, s]
    return torch.stack(starts, 1).reshape(B * S, *h.shape[1:]), h


def _compose_backward(P, e, dhf, S):
    """Incoming state gradient of every segment (B * S, H, D, D) and the
    gradient at the sequence start, in float64."""
    B = P.shape[0] // S
    P = P.view(B, S, *P.shape[1:]).double()
    e = e.view(B, S, *e.shape[1:]).double()
    g = dhf.double()
    g_in = [None] * S
    for s in range(S - 1, -1, -1):
        g_in[s] = g
        g = P[:, s].transpose(-1, -2) @ g + e[:, s]
    return torch.stack(g_in, 1).reshape(B * S, *g.shape[1:]), g


def segmented_forward(q, k, v, w, b, g, scale, h0, S):
    """Forward with every sequence cut into S segments.  Returns
    (o, h_final, state), or None when a state sanitiser acted (the caller
    then runs the serial path)."""
    B, T, H, D = q.shape
    xs = [_split(t, S) for t in (q, k, v, w, b, g)]
    st, P, c = _sp.sp_forward_local(*xs, scale, 0)
    p = st.p
    h0 = torch.zeros((B, H, D, D), device=p.dev) if h0 is None else \
        torch.as_tensor(h0).to(p.dev, torch.float32)
    starts, hf = _compose_forward(P, c, h0, S)
    st.h_start = starts.float().contiguous()
    h_end = torch.empty_like(st.h_start)
    _sp._seg(1, st.ws, p, st.h_start, st.o, h_end)
    bits = st.bits | _lib.workspace_status(st.ws, p.stream)
    if bits & _lib.STATUS_WAIT_TIMEOUT:
        raise _lib.Gdn2Error("segmented forward: a bounded barrier wait inside a kernel timed out")
    if bits & _lib.STATUS_FWD_STATE_CLIPPED:
        return None
    return st.o.view(B, T, H, D), hf.float(), SegmentedState(st, S, B, P)


def segmented_backward(state, dout, dh_final):
    """(dq, dk, dv, dw, db, dg, dh0) of a segmented forward, or None when a
    sanitiser acted on the backward chain (the caller reruns serially)."""
    st, S = state.st, state.S
    p = st.p
    B, T = state.B, p.T * S
    do = _split(torch.as_tensor(dout).to(p.dev, torch.float32).contiguous(), S)
    e = _sp.sp_backward_local(st, do)
    dhf = torch.zeros((B, p.H, p.D, p.D), device=p.dev) if dh_final is None else \
        torch.as_tensor(dh_final).to(p.dev, torch.float32)
    g_in, g0 = _compose_backward(state.maps, e, dhf, S)
    grads = _bwd.gdn2_backward(*p.t, p.scale, st.h_start, st.do, g_in.float().contiguous(),
                               workspace=st.ws, _prep_done=True)
    bits = st.bwd_bits | _lib.workspace_status(st.ws, p.stream)
    if bits & _lib.STATUS_WAIT_TIMEOUT:
        raise _lib.Gdn2Error("segmented backward: a bounded barrier wait inside a kernel timed out")
    if bits & (_lib.STATUS_BWD_STATE_CLIPPED | _lib.STATUS_EXACT_RECOMPUTE):
        return None
    out = [t.reshape(B, T, p.H, p.D).to(dt) for t, dt in zip(grads[:6], p.in_dtypes)]
    dh0 = torch.nan_to_num(g0.clamp(-_FINAL_CLIP, _FINAL_CLIP), nan=0.0).float()
    return (*out, dh0)


class _SegCore(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, w, b, g, h0, scale, S):
        from . import gdn2_pipeline as _pipe
        r = segmented_forward(q, k, v, w, b, g, scale, h0, S)
        ctx.scale, ctx.state = scale, None
        if r is None:   # a clip acted: the serial path, residuals kept
            (o, hf), res = _pipe._gdn2_core_fwd(q, k, v, w, b, g, scale, h0)
            ctx.ws = res[7]
        else:
            o, hf, ctx.state = r
            ctx.ws = None
        ctx.save_for_backward(q, k, v, w, b, g, h0)
        return o, hf

    @staticmethod
    def backward(ctx, do, dhf):
        q, k, v, w, b, g, h0 = ctx.saved_tensors
        if do is None:
            do = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        grads = None
        if ctx.state is not None:
            grads = segmented_backward(ctx.state, do, dhf)
        if grads is None:   # serial backward (recomputes the forward without residuals)
            grads = _bwd.gdn2_backward(q, k, v, w, b, g, ctx.scale, h0, do, dhf,
                                       workspace=ctx.ws)
        ctx.state = ctx.ws = None
        return (*grads, None, None)


def gdn2_segmented_forward_trainable(q, k, v, w, b, g, scale, h0=None, segments=None):
    """``gdn2_pallas_forward_trainable`` with the chunk-parallel scan: every
    sequence runs as ``segments`` time segments (default: plan_segments for
    this GPU).  Needs BT = D = 128 and T a multiple of segments * BT; falls
    back to the serial path per call whenever a state sanitiser acts."""
    B, T, H, D = q.shape
    if segments is None:   # planned: only the BT = D = 128 path has the segment joins
        sms = torch.cuda.get_device_properties(q.device).multi_processor_count
        segments = plan_segments(B, T, H, _fwd.BT, sms) if int(_fwd.BT) == 128 and D == 128 else 1
    if h0 is None:
        h0 = torch.zeros((B, H, D, D), dtype=torch.float32, device=q.device)
    if segments <= 1:
        from . import gdn2_pipeline as _pipe
        return _pipe.gdn2_pallas_forward_trainable(q, k, v, w, b, g, scale, h0)
    if T % (segments * _fwd.BT):
        raise _fwd.Gdn2ShapeError(f"T = {T} is not a multiple of segments x BT")
    return _SegCore.apply(q, k, v, w, b, g, h0, float(scale), int(segments))
