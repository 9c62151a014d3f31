"""Forward + backward of host-resident batches, streamed through the GPU.

``gdn2_fwd_bwd(q, k, v, w, b, g, scale, dout, dh_final, h0=None)`` returns
``(o, h_final, (dq, dk, dv, dw, db, dg, dh0))``: the outputs of
``gdn2_pallas_forward`` and the cotangents that ``_gdn2_core_bwd`` returns
for (dout, dh_final) (gdn2_pipeline.py:64-137), i.e. one training step of the
layer in a single call.

With CUDA tensors it runs the forward (keeping its per-chunk residuals) and
the backward on the current stream.  With host tensors, every (batch, head)
being independent (gdn2_fwd.py:154), the batch is cut into (batch rows x
head group) shards that flow through a ring of device buffer sets: the copy of shard s+1 to the device
(one stream), the kernels of the shards in flight (one stream per buffer
set) and the copy of shard s-1 back to the host (one stream) overlap, so the step costs about the larger of the PCIe traffic and the
compute instead of their sum.  Results equal the unsharded call (the same
kernels run on every (batch, head)).
"""
from __future__ import annotations

import torch

from . import _lib
from . import gdn2_fwd as _fwd

NAMES = ("q", "k", "v", "w", "b", "g")


class _Slot:
    """Device buffers of one in-flight shard."""

    def __init__(self, p, Bs, dev, with_h0, backward):
        T, H, D = p.T, p.H, p.D
        shp, st = (Bs, T, H, D), (Bs, H, D, D)
        f32 = torch.float32
        self.x = [torch.empty(shp, dtype=p.dtype, device=dev) for _ in NAMES]
        self.h0 = torch.empty(st, dtype=f32, device=dev) if with_h0 else None
        self.o = torch.empty(shp, dtype=f32, device=dev)
        self.hf = torch.empty(st, dtype=f32, device=dev)
        self.do = torch.empty(shp, dtype=f32, device=dev) if backward else None
        self.dhf = torch.empty(st, dtype=f32, device=dev) if backward else None
        self.g = [torch.empty(shp, dtype=p.dtype, device=dev) for _ in NAMES] if backward else []
        self.dh0 = torch.empty(st, dtype=f32, device=dev) if backward else None
        n = _lib.load().gdn2_workspace_bytes(Bs, T, H, D, p.C, int(backward))
        self.ws = torch.empty(n, dtype=torch.uint8, device=dev)
        self.loaded = torch.cuda.Event()    # inputs on the device
        self.computed = torch.cuda.Event()  # outputs ready, inputs free
        self.drained = torch.cuda.Event()   # outputs copied to the host


def _run(p, lib, code, xs, h0, do, dhf, o, hf, grads, dh0, ws, Bs, stream):
    """gdn2_fwd (keeping residuals when a backward follows), then gdn2_bwd
    unless ``do`` is None, on `stream`."""
    ptr = lambda t: t.data_ptr() if t is not None else None
    bwd = do is not None
    rc = lib.gdn2_fwd(code, *[t.data_ptr() for t in xs], ptr(h0), o.data_ptr(), hf.data_ptr(),
                      ws.data_ptr(), ws.numel(), int(bwd), Bs, p.T, p.H, p.D, p.C, p.bc, p.scale,
                      p.clip, stream)
    _lib.check(rc, "gdn2_fwd")
    if not bwd:
        return
    rc = lib.gdn2_bwd(code, *[t.data_ptr() for t in xs], ptr(h0), do.data_ptr(), dhf.data_ptr(),
                      *[t.data_ptr() for t in grads], dh0.data_ptr(), ws.data_ptr(), ws.numel(), 1,
                      Bs, p.T, p.H, p.D, p.C, p.bc, p.scale, p.clip, stream)
    _lib.check(rc, "gdn2_bwd")


def _shard_plan(B, H, Bs, Hs, edges):
    """Shards (b0, h0, heads) in streaming order: batch rows of Bs by head
    groups of Hs; with ``edges`` the first and the last group go as single
    heads (the copy-in before the first kernels and the work after the last
    copy-in are what the pipeline cannot overlap)."""
    plan = [(bi * Bs, gi * Hs, Hs) for bi in range(B // Bs) for gi in range(H // Hs)]
    if edges and Hs > 1 and len(plan) > 2:
        first, last = plan[0], plan[-1]
        plan = ([(first[0], first[1] + i, 1) for i in range(Hs)] + plan[1:-1]
                + [(last[0], last[1] + i, 1) for i in range(Hs)])
    return plan


def _head_group(Bs, T, H, D=128):
    """Smallest head group whose shard still gives the chunk kernels one CTA
    per SM (148 on a B200): small shards shorten the copy-in of the first
    shard and the copy-out of the last, which nothing overlaps."""
    nc = max(1, T // _fwd._kernel_chunk(T, int(_fwd.BT), D))
    for hs in range(1, H + 1):
        if H % hs == 0 and Bs * hs * nc >= 148:
            return hs
    return H


def gdn2_fwd_bwd(q, k, v, w, b, g, scale, dout=None, dh_final=None, h0=None, shard=1, depth=3,
                 out=None, heads=None, edges=True):
    """Forward and backward of one layer call (forward only when ``dout`` is
    None; a missing ``dh_final`` is zero).  Host tensors (pinned for
    asynchronous copies) are streamed in shards of ``shard`` batch rows by
    ``heads`` heads (default: the smallest group that fills the GPU), each
    tensor moved by one pitched copy, with ``depth`` shards in flight
    (``edges``: the first and the last head group go as single heads, which
    shortens the copy-in before the first kernels and the work after the
    last copy-in); ``out`` may hold preallocated host outputs
    ``(o, h_final[, dq, dk, dv, dw, db, dg, dh0])``.  Gradients come back in
    the input dtype, o / h_final / dh0 in float32; the gradient tuple is None
    for a forward only."""
    xs = [torch.as_tensor(t).contiguous() for t in (q, k, v, w, b, g)]
    bwd = dout is not None
    if xs[0].device.type == "cuda":
        p = _fwd._Prepared(*xs, scale, h0)
        lib = _lib.load()
        ws = p.workspace(bwd)
        o = torch.empty((p.B, p.T, p.H, p.D), dtype=torch.float32, device=p.dev)
        hf = torch.empty((p.B, p.H, p.D, p.D), dtype=torch.float32, device=p.dev)
        do = dhf = dh0 = None
        grads = []
        if bwd:
            do = torch.as_tensor(dout).to(p.dev, torch.float32).contiguous()
            dhf = torch.zeros_like(hf) if dh_final is None else \
                torch.as_tensor(dh_final).to(p.dev, torch.float32).contiguous()
            grads = [torch.empty_like(t) for t in p.t]
            dh0 = torch.empty((p.B, p.H, p.D, p.D), dtype=torch.float32, device=p.dev)
        _run(p, lib, p.code, p.t, p.h0, do, dhf, o, hf, grads, dh0, ws, p.B, p.stream)
        return o, hf, ((*grads, dh0) if bwd else None)

    B, T, H, D = xs[0].shape
    dt = xs[0].dtype
    if dt not in (torch.float32, torch.bfloat16) or any(t.dtype != dt for t in xs):
        raise _fwd.Gdn2ShapeError("streamed inputs must share one dtype, float32 or bfloat16")
    if T % int(_fwd.BT):
        raise _fwd.Gdn2ShapeError(f"L={T} must be divisible by BT={_fwd.BT}.")
    do_h = dhf_h = None
    if bwd:
        do_h = torch.as_tensor(dout).float().contiguous()
        if dh_final is not None:
            dhf_h = torch.as_tensor(dh_final).float().contiguous()
    h0_h = None if h0 is None else torch.as_tensor(h0).float().contiguous()
    Bs = max(1, min(int(shard), B))
    if B % Bs:
        raise _fwd.Gdn2ShapeError(f"shard={Bs} must divide the batch B={B}")
    Hs = _head_group(Bs, T, H, D) if heads is None else max(1, min(int(heads), H))
    if H % Hs:
        raise _fwd.Gdn2ShapeError(f"heads={Hs} must divide the head count H={H}")
    dev = torch.device("cuda", torch.cuda.current_device())
    # constants and chunking are validated exactly as for the device path
    no_pair = _fwd.GATES == "activated" and bool((xs[5] > 0).any())

    def prepared(hs):
        pp = _fwd._Prepared(*[torch.zeros((Bs, T, hs, D), dtype=dt, device=dev)] * 6, scale,
                            None if h0_h is None else torch.empty((Bs, hs, D, D), device=dev))
        if pp.C == 64 and D == 128 and T % 128 == 0 and no_pair:
            pp.code |= _lib.NO_PAIR   # as _Prepared decides for device tensors
        return pp

    p = prepared(Hs)
    lib = _lib.load()
    if out is None:
        pin = torch.cuda.is_available()
        mk = lambda s, d: torch.empty(s, dtype=d, pin_memory=pin)
        out = (mk((B, T, H, D), torch.float32), mk((B, H, D, D), torch.float32))
        if bwd:
            out += (*[mk((B, T, H, D), dt) for _ in NAMES], mk((B, H, D, D), torch.float32))
    if any(not t.is_contiguous() for t in out):
        raise _fwd.Gdn2ShapeError("preallocated host outputs must be contiguous")
    o_h, hf_h, *g_h = out
    dh0_h = g_h.pop() if bwd else None
    nb, nhg = B // Bs, H // Hs
    plan = _shard_plan(B, H, Bs, Hs, edges)
    preps = {hs: (p if hs == Hs else prepared(hs)) for hs in {x[2] for x in plan}}
    nsh = len(plan)
    nslot = max(1, min(int(depth), nsh))
    slots = [_Slot(p, Bs, dev, h0_h is not None, bwd) for _ in range(nslot)]
    # each shard's status header (gdn2_workspace_status) lands in pinned memory
    status_h = torch.zeros((nsh, 5), dtype=torch.int32, pin_memory=True)
    # one compute stream per slot: the kernels of consecutive shards overlap,
    # which hides the latency of the chunk scans (sequential over a shard's
    # chunks, so a small shard leaves most SMs idle while they run)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_runs = [torch.cuda.Stream(dev) for _ in range(nslot)]
    cur = torch.cuda.current_stream(dev)
    for st in (s_in, s_out, *s_runs):
        st.wait_stream(cur)

    def copy(host, devt, b0, h0, hs, seq, to_device, stream):
        # one pitched DMA per tensor: rows (b, t) of the shard, heads h0 .. h0+hs-1
        # (a shard of fewer heads than the slot uses the slot buffers' prefix)
        eb = host.element_size()
        head = (D if seq else D * D) * eb
        rows = Bs * (T if seq else 1)
        hp = host.data_ptr() + b0 * (T if seq else 1) * H * head
        _lib.check(lib.gdn2_copy_heads(hp, devt.data_ptr(), rows, H, h0, hs, head, int(to_device),
                                       stream.cuda_stream), "gdn2_copy_heads")

    for s in range(nsh):
        sl = slots[s % nslot]
        b0, h0s, hs = plan[s]
        ps = preps[hs]
        if s >= nslot:
            s_in.wait_event(sl.computed)        # the kernels of shard s - nslot read these
        for dst, src in zip(sl.x, xs):
            copy(src, dst, b0, h0s, hs, True, True, s_in)
        if bwd:
            copy(do_h, sl.do, b0, h0s, hs, True, True, s_in)
            if dhf_h is None:
                with torch.cuda.stream(s_in):
                    sl.dhf.zero_()
            else:
                copy(dhf_h, sl.dhf, b0, h0s, hs, False, True, s_in)
        if sl.h0 is not None:
            copy(h0_h, sl.h0, b0, h0s, hs, False, True, s_in)
        sl.loaded.record(s_in)
        s_run = s_runs[s % nslot]
        s_run.wait_event(sl.loaded)
        if s >= nslot:
            s_run.wait_event(sl.drained)            # outputs of shard s - nslot copied out
        _run(ps, lib, ps.code, sl.x, sl.h0, sl.do, sl.dhf, sl.o, sl.hf, sl.g, sl.dh0, sl.ws, Bs,
             s_run.cuda_stream)
        with torch.cuda.stream(s_run):
            off = (sl.ws.data_ptr() + 255) // 256 * 256 - sl.ws.data_ptr()
            status_h[s].copy_(sl.ws[off:off + 20].view(torch.int32), non_blocking=True)
        sl.computed.record(s_run)
        s_out.wait_event(sl.computed)
        copy(o_h, sl.o, b0, h0s, hs, True, False, s_out)
        copy(hf_h, sl.hf, b0, h0s, hs, False, False, s_out)
        for dst, src in zip(g_h, sl.g):
            copy(dst, src, b0, h0s, hs, True, False, s_out)
        if bwd:
            copy(dh0_h, sl.dh0, b0, h0s, hs, False, False, s_out)
        sl.drained.record(s_out)
    s_out.synchronize()
    for st in s_runs:
        st.synchronize()
    st = status_h.any(dim=0).tolist()
    _lib.LAST_STATUS = sum(bit for bit, on in zip(
        (_lib.STATUS_WAIT_TIMEOUT, _lib.STATUS_FWD_STATE_CLIPPED, _lib.STATUS_BWD_STATE_CLIPPED,
         _lib.STATUS_EXACT_RECOMPUTE, _lib.STATUS_B4_EXACT), st) if on)
    if _lib.CHECK_STATUS != "never" and _lib.LAST_STATUS & _lib.STATUS_WAIT_TIMEOUT:
        raise _lib.Gdn2Error("gdn2_fwd_bwd: a bounded barrier wait inside a kernel timed out; "
                             "the results of this call are invalid")
    return o_h, hf_h, ((*g_h, dh0_h) if bwd else None)
