"""Sequence parallelism for long sequences (one process per GPU).

Each rank owns one contiguous time segment of every (batch, head).  The
inter-chunk recurrence is affine (h <- M_c h + B_c, see csrc/gdn2_tc_kernels.cu),
so a segment acts on its start state as  h_end = P h_start + c  with
P = M_last ... M_first.  The reference runs the scan serially over the whole
sequence (gdn2_fwd.py:362, gdn2_bwd.py:77); here:

  forward   1. every rank runs its segment from a zero state  -> c, residuals
            2. every rank forms P (gdn2_sp_segment op 0)
            3. all ranks exchange (P, c): two D x D tiles per (batch, head)
            4. each rank composes its start state in float64 and rescans
               (op 1) -> o, per-chunk states; the last segment's end state is
               h_final
  backward  the gradient flows the other way: g_start = P^T g_end + e, with e
            the segment's start gradient for a zero incoming one (op 2); the
            ranks exchange e, compose their incoming gradient and run the
            ordinary backward of their segment with it.

Exactness.  The reference sanitises the state after every chunk (h and dh
clipped to +-CLIP, gdn2_fwd.py:358, gdn2_bwd.py:73) and dv_new inside the
backward chain (gdn2_bwd.py:68).  A clip that acts makes a segment's map
non-affine, so the composed start states (and gradients) are exact only while
no sanitiser acts on the chain.  The kernels report every such event in the
workspace status (STATUS_*_STATE_CLIPPED, STATUS_EXACT_RECOMPUTE); the ranks
exchange these bits and raise Gdn2SaturationError instead of returning
inexact results.  Within one rank (and in the non-parallel entry points) the
sanitisers are applied exactly.

Only these D x D boundary tiles cross the interconnect.  The exchange is one
all-gather through `torch.distributed` (NCCL over NVLink on B200 nodes); a
custom `gather(list_of_tensors) -> list_per_rank` can replace it, which is how
the tests emulate several ranks on one device.
"""
from __future__ import annotations

import torch

from . import _lib
from . import gdn2_fwd as _fwd


class Gdn2SaturationError(_lib.Gdn2Error):
    """A state sanitiser acted inside a segment, so the affine composition of
    the segments would not equal the reference's serial scan."""


def _status(p, ws):
    return _lib.workspace_status(ws, p.stream)


def _check_linear(bits, p, gather, what):
    """All ranks share their status bits; raise if any rank saw a clip that
    breaks the segment maps, or a timed-out wait."""
    t = torch.tensor([bits], dtype=torch.int32, device=p.dev)
    allbits = 0
    for x in gather(t):
        allbits |= int(x.item())
    if allbits & _lib.STATUS_WAIT_TIMEOUT:
        raise _lib.Gdn2Error(f"{what}: a bounded barrier wait inside a kernel timed out")
    bad = _lib.STATUS_FWD_STATE_CLIPPED if what == "sp_forward" else \
        (_lib.STATUS_BWD_STATE_CLIPPED | _lib.STATUS_EXACT_RECOMPUTE)
    if allbits & bad:
        raise Gdn2SaturationError(
            f"{what}: the CLIP sanitiser acted on the recurrence inside a segment "
            f"(status bits {allbits:#x}); the sequence-parallel composition is exact only "
            "while it does not; run this input without sequence parallelism")


def compose_forward(maps, consts, h0):
    """Start state of every segment and the final state, in float64:
    h_start[0] = h0, h_start[r+1] = maps[r] h_start[r] + consts[r]."""
    h = h0.double()
    starts = []
    for P, c in zip(maps, consts):
        starts.append(h)
        h = P.double() @ h + c.double()
    return starts, h


def compose_backward(maps, terms, g_final):
    """Incoming gradient of every segment and the gradient at the sequence
    start: g_in[R-1] = g_final, g_in[r-1] = maps[r]^T g_in[r] + terms[r]."""
    g = g_final.double()
    g_in = [None] * len(maps)
    for r in range(len(maps) - 1, -1, -1):
        g_in[r] = g
        g = maps[r].double().transpose(-1, -2) @ g + terms[r].double()
    return g_in, g


def dist_gather(group=None):
    """all-gather of one tensor per rank through torch.distributed."""
    import torch.distributed as dist

    def gather(t):
        out = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
        dist.all_gather(out, t.contiguous(), group=group)
        return out

    return gather


def _seg(op, ws, p, inp, o, out):
    rc = _lib.load().gdn2_sp_segment(
        op, ws.data_ptr(), ws.numel(), inp.data_ptr() if inp is not None else None,
        o.data_ptr() if o is not None else None, out.data_ptr(), p.B, p.T, p.H, p.D, p.C, p.bc,
        p.scale, p.clip, p.stream)
    _lib.check(rc, "gdn2_sp_segment")


class SegmentState:
    """Residuals of one rank's segment kept between forward and backward."""

    def __init__(self, p, ws, maps, rank, h_start):
        self.p, self.ws, self.maps, self.rank, self.h_start = p, ws, maps, rank, h_start


def sp_forward_local(q, k, v, w, b, g, scale, rank):
    """Steps 1-2 of the forward on this rank's (B, T/R, H, D) segment: returns
    (state, P, c) where P, c (B, H, D, D) are the segment's affine map."""
    p = _fwd._Prepared(q, k, v, w, b, g, scale, None)
    if not (p.C == 128 and p.D == 128):
        raise _fwd.Gdn2ShapeError("sequence parallelism needs BT = D = 128")
    if p.T != p.T_user:
        raise _fwd.Gdn2ShapeError("sequence parallelism needs segments divisible by BT")
    ws = p.workspace(True)
    # o is formed by the rescan (op 1), not by this zero-state run
    o, c_seg, _ = _fwd._run_forward(p, save_residuals=True, ws=ws, outputs=False)
    bits = _status(p, ws)
    P = torch.empty((p.B, p.H, p.D, p.D), dtype=torch.float32, device=p.dev)
    _seg(0, ws, p, None, None, P)
    st = SegmentState(p, ws, None, rank, None)
    st.o = o
    st.bits = bits
    return st, P, c_seg


def sp_forward_finish(state, maps, consts, h0=None):
    """Step 4: compose this rank's start state from every rank's (P, c) and
    rescan.  Returns (o_local, h_final)."""
    p = state.p
    h0 = torch.zeros((p.B, p.H, p.D, p.D), device=p.dev) if h0 is None else \
        torch.as_tensor(h0).to(p.dev, torch.float32)
    starts, final = compose_forward(maps, consts, h0)
    state.maps = maps
    state.h_start = starts[state.rank].float().contiguous()
    h_end = torch.empty_like(state.h_start)
    _seg(1, state.ws, p, state.h_start, state.o, h_end)
    state.bits |= _status(p, state.ws)
    return state.o, final.float()


def sp_backward_local(state, dout):
    """The segment's start gradient for a zero incoming gradient (B, H, D, D)."""
    p = state.p
    state.do = torch.as_tensor(dout).to(p.dev, torch.float32).contiguous()
    e = torch.empty((p.B, p.H, p.D, p.D), dtype=torch.float32, device=p.dev)
    _seg(2, state.ws, p, state.do, None, e)
    state.bwd_bits = _status(p, state.ws)
    return e


def sp_backward_finish(state, terms, dh_final=None):
    """Compose this rank's incoming gradient and run its segment backward.
    Returns (dq, dk, dv, dw, db, dg) of the segment and dh0."""
    from . import gdn2_bwd as _bwd
    p = state.p
    dhf = torch.zeros((p.B, p.H, p.D, p.D), device=p.dev) if dh_final is None else \
        torch.as_tensor(dh_final).to(p.dev, torch.float32)
    g_in, g0 = compose_backward(state.maps, terms, dhf)
    g_rank = g_in[state.rank].float().contiguous()
    grads = _bwd.gdn2_backward(*p.t, p.scale, state.h_start, state.do, g_rank, workspace=state.ws,
                               _prep_done=True)
    state.bwd_bits |= _status(p, state.ws)
    grads = [t.to(dt) for t, dt in zip(grads[:6], p.in_dtypes)]
    dh0 = torch.nan_to_num(g0.clamp(-1e4, 1e4), nan=0.0).float()
    return (*grads, dh0)


def sp_forward(q, k, v, w, b, g, scale, h0=None, rank=0, gather=None):
    """Forward of this rank's segment with the exchange through `gather`
    (default: torch.distributed all-gather).  Returns (o_local, h_final, state)."""
    gather = gather or dist_gather()
    st, P, c = sp_forward_local(q, k, v, w, b, g, scale, rank)
    o, hf = sp_forward_finish(st, gather(P), gather(c), h0)
    _check_linear(st.bits, st.p, gather, "sp_forward")
    return o, hf, st


def sp_backward(state, dout, dh_final, gather=None):
    """Backward of this rank's segment; dh0 is the same on every rank."""
    gather = gather or dist_gather()
    e = sp_backward_local(state, dout)
    out = sp_backward_finish(state, gather(e), dh_final)
    _check_linear(state.bwd_bits, state.p, gather, "sp_backward")
    return out


class _SPCore(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, w, b, g, h0, scale, rank, gather):
        o, hf, st = sp_forward(q, k, v, w, b, g, scale, h0, rank, gather)
        ctx.st, ctx.gather = st, gather
        return o, hf

    @staticmethod
    def backward(ctx, do, dhf):
        grads = sp_backward(ctx.st, do, dhf, ctx.gather)
        ctx.st = None
        return (*grads, None, None, None)


def gdn2_sp_forward_trainable(q, k, v, w, b, g, scale, h0=None, group=None):
    """Differentiable sequence-parallel forward over the ranks of `group`
    (default: the world).  Each rank passes its own time segment."""
    import torch.distributed as dist
    rank = dist.get_rank(group)
    B, T, H, D = q.shape
    if h0 is None:
        h0 = torch.zeros((B, H, D, D), dtype=torch.float32, device=q.device)
    return _SPCore.apply(q, k, v, w, b, g, h0, float(scale), rank, dist_gather(group))
