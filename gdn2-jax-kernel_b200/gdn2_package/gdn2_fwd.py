"""GDN-2 chunked forward on B200 (mirrors the reference module gdn2_fwd.py).

Public surface kept from the reference (Akseleu-J/gdn2-jax-kernel):
  * module constants ``BT``, ``BC``, ``MB``, ``CLIP`` (gdn2_fwd.py:29-33), read
    at call time, so ``gdn2_fwd.BT = 128`` takes effect for every later call
    of this package (forward and backward alike);
  * ``gdn2_pallas_forward(q,k,v,w,b,g,scale,h0=None,debug_tag="")`` returning
    ``(o, h_final)`` (gdn2_fwd.py:400-424);
  * ``gdn2_pallas_forward_with_residuals`` (gdn2_fwd.py:427-457).

Arrays are torch tensors (B, T, H, D) in float32 or bfloat16.  CUDA tensors
are computed in place on the current stream; CPU tensors are copied to the
current CUDA device and the results copied back (the host-buffer path).
``o`` and ``h_final`` are float32, as in the reference (gdn2_fwd.py:164-165).
The compute runs in libgdn2.so (hand-written sm_100a kernels); there is no
other backend.
"""
from __future__ import annotations

import os

import torch

from . import _lib

# ---------- constants (gdn2_fwd.py:29-33) ----------
BT = 256     # chunk length
BC = 128     # sub-block length: where the WY solve and B4 sanitise (results depend on it only where a clip acts)
MB = 16      # micro-block of the triangular solve
CLIP = 1e4   # stage sanitiser bound
# Chunk length policy.  EXACT_BT = True (default) runs chunks of BT itself
# (split into 128 or 64 when BT is larger); with BT = 128 or 64 this places
# every clip where the reference places it.  EXACT_BT = False lets a head dim of
# 128 run chunks of 128 (the tensor-core kernels) whenever T allows, whatever
# BT says: the chunked form is exact for any chunk length, so results agree
# to float32 rounding unless a gate is positive and the +-20 exponent clip or
# CLIP saturate (they act per chunk).
EXACT_BT = True
# BT = 64 with D = 128 (and T a multiple of 128) runs on the tensor-core
# kernels, two chunks per 128-row tile computing the same BT = 64 function.
# With a positive log-decay gate (outside -softplus's range; the reference
# tests' all-ones inputs) the chunk states saturate at CLIP and some
# gradients become cancellations of ~CLIP^2-sized products, where the
# 3xTF32 products' relative error (~2^-22 of each term) shows: such calls,
# and PAIR64 = False, run the float32 CUDA-core kernels instead.
PAIR64 = True
# T not a multiple of BT: the reference refuses it (gdn2_fwd.py:145-146), as
# does this module by default.  MASKED_TAIL = True instead pads the sequence
# with zero tokens (g = 0, k = q = v = w = b = 0), which leave the state and
# every output and gradient of the real tokens unchanged, and slices back.
MASKED_TAIL = False

# Gate inputs.  "activated" (the reference's contract, README.md:60-68): the
# caller passes w = sigmoid(.), b = sigmoid(.), g = -softplus(.).  "raw": the
# caller passes the pre-activations, the kernels apply the activations as
# they load w, b, g (no separate pass over them), and the backward returns
# gradients with respect to the pre-activations.
GATES = "activated"

_GDN2_FWD_DIAG = os.environ.get("GDN2_FWD_DIAG", "0") == "1"
_KERNEL_CHUNKS = (128, 64)
_SUPPORTED_D = (64, 128)   # the fused kernels
_STAGE_D = (256,)          # head dims served by the stage kernels alone (BT 64 or 128)


class Gdn2ShapeError(ValueError, AssertionError):
    """Unsupported shape or argument.  Derives from AssertionError too, since
    the reference rejects these with ``assert`` (gdn2_fwd.py:145-146)."""


def _kernel_chunk(T, bt, D):
    """Chunk length the kernels run with for the user's BT.  The chunked form
    is exact for any chunk length: only the +-20 pair-decay clip and CLIP see
    the chunking, and both act on saturated inputs alone.  So a BT of 256 runs
    as chunks of 128, and with EXACT_BT = False a head dim of 128 runs chunks
    of 128 for any BT that divides T (the tensor-core path)."""
    if T % bt != 0:
        raise Gdn2ShapeError(f"L={T} must be divisible by BT={bt}.")
    if not EXACT_BT and D == 128 and T % 128 == 0:
        return 128
    for c in _KERNEL_CHUNKS:
        if bt % c == 0 and T % c == 0 and c <= bt:
            return c
    raise Gdn2ShapeError(f"BT={bt} unsupported: kernels run chunks of 128 or 64")


_LARGE_THRESHOLD = 1e6   # gdn2_fwd.py:38


def _diag_line(tag, n_bad, mx):
    """The reference's two reports (gdn2_fwd.py:56-69), or None."""
    if n_bad:
        return f"[GDN2-FWD-DIAG] non-finite at {tag}: n_nonfinite={n_bad} max_abs={mx:.3e}"
    if mx > _LARGE_THRESHOLD:
        return f"[GDN2-FWD-DIAG] large value at {tag}: max_abs={mx:.3e}"
    return None


def _stage_diag(tag, x):
    """Non-finite / large-value report of one tensor when GDN2_FWD_DIAG=1
    (gdn2_fwd.py:47-76); returns x."""
    if not _GDN2_FWD_DIAG:
        return x
    finite = torch.isfinite(x)
    n_bad = int((~finite).sum())
    mx = float(torch.where(finite, x, torch.zeros_like(x)).abs().max()) if x.numel() else 0.0
    line = _diag_line(tag, n_bad, mx)
    if line:
        print(line)
    return x


def _stage_reports(debug_tag, ws, stream):
    """Per-stage reports of the forward that just ran on ``ws``, from the
    counters its kernels accumulated on the device (every stage the
    reference's gdn2_pallas_forward checks, gdn2_fwd.py:407-417, 360-363)."""
    lines = []
    for tag, (n_bad, mx) in _lib.diag_read(ws, stream).items():
        line = _diag_line(f"{debug_tag}:{tag}", n_bad, mx)
        if line:
            lines.append(line)
            print(line)
    return lines


class _Prepared:
    """Validated, device-resident, contiguous operands of one call."""

    def __init__(self, q, k, v, w, b, g, scale, h0):
        ts = (q, k, v, w, b, g)
        if not all(isinstance(t, torch.Tensor) for t in ts):
            ts = tuple(torch.as_tensor(t) for t in ts)
        shape = tuple(ts[0].shape)
        if len(shape) != 4:
            raise Gdn2ShapeError(f"inputs must be (B, T, H, D); got {shape}")
        for t in ts:
            if tuple(t.shape) != shape:
                raise Gdn2ShapeError(f"all inputs must share shape {shape}; got {tuple(t.shape)}")
        B, T, H, D = shape
        if D not in _SUPPORTED_D:
            raise Gdn2ShapeError(f"head dim D={D} unsupported (64 or 128)")
        self.bt_user = int(BT)
        self.T_user = T
        if MASKED_TAIL and self.bt_user > 0 and T % self.bt_user:
            T = -(-T // self.bt_user) * self.bt_user
        self.B, self.T, self.H, self.D = B, T, H, D
        self.C = _kernel_chunk(T, self.bt_user, D)
        bc = int(BC)
        if bc <= 0 or self.bt_user % bc != 0:
            raise Gdn2ShapeError(f"BC={bc} must divide BT={self.bt_user}")
        if bc % MB:
            raise Gdn2ShapeError(f"BC={bc} must be a multiple of MB={MB} (gdn2_fwd.py:194)")
        # BC places the sanitisers of the WY solve and of B4's accumulators.
        # Chunks merged beyond BT (EXACT_BT = False) already move them, and
        # run with sub-blocks of 64, the tensor-core kernels' fast layout.
        self.bc = bc if self.C % bc == 0 else self.C
        if self.C > self.bt_user:
            self.bc = 64
        if any(not t.dtype.is_floating_point for t in ts):
            raise Gdn2ShapeError("inputs must be floating point")
        if h0 is not None and tuple(torch.as_tensor(h0).shape) != (B, H, D, D):
            raise Gdn2ShapeError(f"h0 must be {(B, H, D, D)}; got {tuple(torch.as_tensor(h0).shape)}")
        self.on_host = ts[0].device.type != "cuda"
        dev = torch.device("cuda", torch.cuda.current_device()) if self.on_host else ts[0].device
        cdt = torch.float32 if any(t.dtype == torch.float32 or t.dtype == torch.float64 for t in ts) \
            else torch.bfloat16
        self.in_dtypes = tuple(t.dtype for t in ts)
        self.dev = dev
        self.dtype = cdt
        self.code = _lib.F32 if cdt == torch.float32 else _lib.BF16
        if GATES not in ("activated", "raw"):
            raise Gdn2ShapeError(f"GATES={GATES!r}: 'activated' or 'raw'")
        if GATES == "raw":
            self.code |= _lib.GATES_RAW
        self.t = tuple(t.to(device=dev, dtype=cdt, non_blocking=True).contiguous() for t in ts)
        if T != self.T_user:
            self.t = tuple(self.pad(t) for t in self.t)
        if self.C == 64 and D == 128 and T % 128 == 0:   # the paired tensor-core tiles apply
            if not PAIR64 or (GATES == "activated" and bool((self.t[5] > 0).any())):
                self.code |= _lib.NO_PAIR
        self.clip = float(CLIP)
        self.scale = float(scale)
        if h0 is None:
            self.h0 = None
            self.h0_dtype = torch.float32
        else:
            h0 = torch.as_tensor(h0)
            self.h0_dtype = h0.dtype
            self.h0 = h0.to(device=dev, dtype=torch.float32, non_blocking=True).contiguous()
        self.stream = torch.cuda.current_stream(dev).cuda_stream

    def pad(self, t):
        """(B, T_user, H, D) -> (B, T, H, D) with zero tokens at the end."""
        if self.T == self.T_user:
            return t
        return torch.nn.functional.pad(t, (0, 0, 0, 0, 0, self.T - self.T_user)).contiguous()

    def unpad(self, t):
        """(B, T, H, D) -> (B, T_user, H, D)."""
        return t if self.T == self.T_user else t[:, :self.T_user].contiguous()

    def ptrs(self):
        return [t.data_ptr() for t in self.t]

    def workspace(self, with_backward):
        n = _lib.load().gdn2_workspace_bytes(self.B, self.T, self.H, self.D, self.C,
                                             int(with_backward))
        if n == 0:
            raise Gdn2ShapeError("invalid sizes for the workspace")
        return torch.empty(n, dtype=torch.uint8, device=self.dev)


def _run_forward(p, save_residuals=False, ws=None, debug_tag="", outputs=True):
    """gdn2_fwd on prepared inputs.  outputs=False (BT = D = 128, residuals
    kept): o is left unwritten for a gdn2_sp_segment op 1 rescan to form."""
    lib = _lib.load()
    lib.gdn2_diag_enable(int(_GDN2_FWD_DIAG))
    o = torch.empty((p.B, p.T, p.H, p.D), dtype=torch.float32, device=p.dev)
    h_final = torch.empty((p.B, p.H, p.D, p.D), dtype=torch.float32, device=p.dev)
    if ws is None:
        ws = p.workspace(save_residuals)
    code = p.code | (0 if outputs else _lib.NO_OUT)
    rc = lib.gdn2_fwd(code, *p.ptrs(), p.h0.data_ptr() if p.h0 is not None else None,
                      o.data_ptr(), h_final.data_ptr(), ws.data_ptr(), ws.numel(),
                      int(save_residuals), p.B, p.T, p.H, p.D, p.C, p.bc, p.scale, p.clip,
                      p.stream)
    _lib.check(rc, "gdn2_fwd")
    _lib.check_status(ws, p.stream, "gdn2_fwd", synced=p.on_host)
    if _GDN2_FWD_DIAG:
        _stage_reports(debug_tag, ws, p.stream)
    return p.unpad(o), h_final, ws


def gdn2_pallas_forward(q, k, v, w, b, g, scale, h0=None, debug_tag=""):
    """Full forward: Kernels A -> B -> C -> D.  Returns o (B,T,H,D) float32
    and h_final (B,H,D,D) float32 (gdn2_fwd.py:400-424)."""
    if _head_dim(q) in _STAGE_D:
        o, h_final, _ = _stage_forward(q, k, v, w, b, g, scale, h0, debug_tag)
        on_host = torch.as_tensor(q).device.type != "cuda"
        return (o.cpu(), h_final.cpu()) if on_host else (o, h_final)
    p = _Prepared(q, k, v, w, b, g, scale, h0)
    o, h_final, _ = _run_forward(p, debug_tag=debug_tag)
    if p.on_host:
        return o.cpu(), h_final.cpu()
    return o, h_final


def _unpack_residuals(p, ws):
    """Views of the residual tiles a forward left in `ws`, in the reference's
    (B, H, nc, ...) layouts (see csrc/gdn2_ws.cuh for the offsets)."""
    B, H, D, C = p.B, p.H, p.D, p.C
    nc = p.T // C
    n = B * H * nc
    base = (ws.data_ptr() + 255) // 256 * 256 - ws.data_ptr() + 256   # after the status word
    f = ws[base:].view(torch.float32)
    sizes = [("AqkT", C * C), ("AT", C * C), ("WT", C * D), ("U", C * D), ("kg", C * D),
             ("qgT", C * D), ("gc", C * D), ("gcl", D), ("hpre", D * D), ("vnew", C * D)]
    out, o = {}, 0
    for name, per in sizes:
        out[name] = f[o:o + per * n]
        o += per * n
    sh = lambda x, *s: x.view(B, H, nc, *s)
    return dict(
        Aqk=sh(out["AqkT"], C, C).transpose(-1, -2),
        A=sh(out["AT"], C, C).transpose(-1, -2),
        w_pseudo=sh(out["WT"], D, C).transpose(-1, -2),
        u=sh(out["U"], C, D), kg=sh(out["kg"], C, D),
        qg=sh(out["qgT"], D, C).transpose(-1, -2),
        gc=sh(out["gc"], C, D), gc_last=sh(out["gcl"], D),
        h_pre_all=sh(out["hpre"], D, D), v_new_all=sh(out["vnew"], C, D))


def gdn2_pallas_forward_with_residuals(q, k, v, w, b, g, scale, h0=None, debug_tag=""):
    """Forward that also returns the per-chunk intermediates (gdn2_fwd.py:427-457):
    Aqk, A, w_pseudo, u, kg, qg, gc_last, h_pre_all, v_new_all, all float32 in
    the batch-major (B, H, nc, ...) layout the backward consumes.  The
    reference additionally returns Akk, which the fused kernels never store."""
    if _head_dim(q) in _STAGE_D:
        o, h_final, res = _stage_forward(q, k, v, w, b, g, scale, h0, debug_tag, residuals=True)
        if torch.as_tensor(q).device.type != "cuda":
            return o.cpu(), h_final.cpu(), {n: t.cpu() for n, t in res.items()}
        return o, h_final, res
    p = _Prepared(q, k, v, w, b, g, scale, h0)
    p.code |= _lib.NO_PAIR   # the residual views below follow the one-chunk tile layout
    o, h_final, ws = _run_forward(p, save_residuals=True, debug_tag=debug_tag)
    res = {n: t.clone() for n, t in _unpack_residuals(p, ws).items()}
    if p.on_host:
        return o.cpu(), h_final.cpu(), {n: t.cpu() for n, t in res.items()}
    return o, h_final, res


# ---------- the reference's stage functions (Kernels A-D, gdn2_fwd.py:142-397) ----------
# Separate entry points on the reference's chunked layouts, for code that
# composes the stages itself (gdn2_pipeline.py:14-31 imports them).  Each runs
# one CUDA kernel of libgdn2.so (gdn2_stage_*); the fused forward above does
# not use them.  BT, BC, CLIP are read at call time; BT is 64, 128 or 256.

def _stage_bt():
    bt = int(BT)
    if bt not in (64, 128, 256):
        raise Gdn2ShapeError(f"the stage functions run BT = 64, 128 or 256; got BT={bt}")
    return bt


def _stage_in(ts):
    """Device, common compute dtype (float32 or bfloat16) and the C code."""
    ts = [torch.as_tensor(t) for t in ts]
    dev = next((t.device for t in ts if t.device.type == "cuda"),
               torch.device("cuda", torch.cuda.current_device()))
    cdt = torch.bfloat16 if all(t.dtype == torch.bfloat16 for t in ts) else torch.float32
    out = [t.to(device=dev, dtype=cdt).contiguous() for t in ts]
    return out, (_lib.BF16 if cdt == torch.bfloat16 else _lib.F32), dev


def _f32(t, dev):
    return torch.as_tensor(t).to(device=dev, dtype=torch.float32).contiguous()


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _check_seq(q):
    B, L, H, D = q.shape
    if D not in _SUPPORTED_D + _STAGE_D:
        raise Gdn2ShapeError(f"head dim D={D} unsupported (64, 128 or 256)")
    bt = _stage_bt()
    if D in _STAGE_D and bt == 256:
        raise Gdn2ShapeError(f"D={D} runs BT = 64 or 128; got BT={bt}")
    if L % bt:
        raise Gdn2ShapeError(f"L={L} must be divisible by BT={bt}.")
    return B, L, H, D, bt


def build_chunk_scores_pallas(q, k, b, g, scale):
    """Kernel A: Aqk, Akk of shape (B, H, n_chunks, BT, BT) (gdn2_fwd.py:142-170)."""
    B, L, H, D, bt = _check_seq(torch.as_tensor(q))
    (q, k, b, g), code, dev = _stage_in((q, k, b, g))
    nc = L // bt
    aqk = torch.empty((B, H, nc, bt, bt), dtype=torch.float32, device=dev)
    akk = torch.empty_like(aqk)
    rc = _lib.load().gdn2_stage_scores(code, q.data_ptr(), k.data_ptr(), b.data_ptr(),
                                       g.data_ptr(), aqk.data_ptr(), akk.data_ptr(), B, L, H, D,
                                       bt, float(scale), float(CLIP), _stream(dev))
    _lib.check(rc, "build_chunk_scores_pallas")
    return aqk, akk


def wy_solve_pallas(Akk):
    """Kernel B: A = (I + Akk)^-1 per chunk (gdn2_fwd.py:246-260).  The
    sub-block level is the reference's block substitution for any number of
    BC sub-blocks (the reference hard-codes two)."""
    bt = _stage_bt()
    Akk = torch.as_tensor(Akk)
    if tuple(Akk.shape[-2:]) != (bt, bt):
        raise Gdn2ShapeError(f"Akk must end in (BT, BT) = {(bt, bt)}")
    dev = Akk.device if Akk.device.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    akk = _f32(Akk, dev)
    a = torch.empty_like(akk)
    n = akk.numel() // (bt * bt)
    bc = int(BC)
    scr = torch.empty((n, bc, bc), dtype=torch.float32, device=dev) if bt == 256 else None
    rc = _lib.load().gdn2_stage_wy_solve(akk.data_ptr(), a.data_ptr(),
                                         scr.data_ptr() if scr is not None else None, n, bt, bc,
                                         float(CLIP), _stream(dev))
    _lib.check(rc, "wy_solve_pallas")
    return a


def recompute_wy_pallas(q, k, v, w, b, g, A):
    """Kernel C: w_pseudo, u, kg, qg (B, H, nc, BT, D) and gc_last (B, H, nc, D)
    (gdn2_fwd.py:298-330)."""
    B, L, H, D, bt = _check_seq(torch.as_tensor(q))
    (q, k, v, w, b, g), code, dev = _stage_in((q, k, v, w, b, g))
    nc = L // bt
    a = _f32(A, dev)
    if tuple(a.shape) != (B, H, nc, bt, bt):
        raise Gdn2ShapeError(f"A must be {(B, H, nc, bt, bt)}")
    shp = (B, H, nc, bt, D)
    wp, u, kg, qg = (torch.empty(shp, dtype=torch.float32, device=dev) for _ in range(4))
    gcl = torch.empty((B, H, nc, D), dtype=torch.float32, device=dev)
    rc = _lib.load().gdn2_stage_recompute_wy(
        code, q.data_ptr(), k.data_ptr(), v.data_ptr(), w.data_ptr(), b.data_ptr(), g.data_ptr(),
        a.data_ptr(), wp.data_ptr(), u.data_ptr(), kg.data_ptr(), qg.data_ptr(), gcl.data_ptr(),
        B, L, H, D, bt, float(CLIP), _stream(dev))
    _lib.check(rc, "recompute_wy_pallas")
    return wp, u, kg, qg, gcl


def _combine(Aqk, w_pseudo, u, kg, qg, gc_last, scale, h0, with_state, debug_tag):
    wp = torch.as_tensor(w_pseudo)
    dev = wp.device if wp.device.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    B, H, nc, bt, D = wp.shape
    if D not in _SUPPORTED_D + _STAGE_D or bt not in (64, 128, 256):
        raise Gdn2ShapeError(f"unsupported chunk tiles {tuple(wp.shape)}")
    xs = [_f32(t, dev) for t in (Aqk, w_pseudo, u, kg, qg, gc_last)]
    h0 = None if h0 is None else _f32(h0, dev)
    o = torch.empty((B, H, nc, bt, D), dtype=torch.float32, device=dev)
    hf = torch.empty((B, H, D, D), dtype=torch.float32, device=dev)
    hpre = torch.empty((nc, B, H, D, D), dtype=torch.float32, device=dev) if with_state else None
    vall = torch.empty((nc, B, H, bt, D), dtype=torch.float32, device=dev) if with_state else None
    ptr = lambda t: t.data_ptr() if t is not None else None
    rc = _lib.load().gdn2_stage_combine(*[t.data_ptr() for t in xs], ptr(h0), o.data_ptr(),
                                        hf.data_ptr(), ptr(hpre), ptr(vall), B, H, nc, bt, D,
                                        float(scale), float(CLIP), _stream(dev))
    _lib.check(rc, "gdn2_inter_chunk_combine")
    _stage_diag(f"{debug_tag}:kernel_D_h_final", hf)
    _stage_diag(f"{debug_tag}:kernel_D_o", o)
    return (o, hf, hpre, vall) if with_state else (o, hf)


def gdn2_inter_chunk_combine(Aqk, w_pseudo, u, kg, qg, gc_last, scale, h0=None, debug_tag=""):
    """Kernel D: o (B, H, nc, BT, D) and h_final (gdn2_fwd.py:338-366)."""
    return _combine(Aqk, w_pseudo, u, kg, qg, gc_last, scale, h0, False, debug_tag)


def gdn2_inter_chunk_combine_with_state(Aqk, w_pseudo, u, kg, qg, gc_last, scale, h0=None,
                                        debug_tag=""):
    """Kernel D that also returns h_pre_all (nc, B, H, D, D) and v_new_all
    (nc, B, H, BT, D), chunk-major as the reference's scan stacks them
    (gdn2_fwd.py:369-397)."""
    return _combine(Aqk, w_pseudo, u, kg, qg, gc_last, scale, h0, True, debug_tag)


# ---------- head dims beyond the fused kernels (D = 256) ----------

def _head_dim(q):
    shape = tuple(torch.as_tensor(q).shape)
    return shape[-1] if len(shape) == 4 else None


def _stage_forward(q, k, v, w, b, g, scale, h0=None, debug_tag="", residuals=False):
    """Forward of a head dim the fused kernels do not cover (D = 256, beyond
    the reference's D = 128, gdn2_fwd.py:145): the reference's own
    composition of Kernels A-D (gdn2_fwd.py:400-457) on the stage kernels.
    Returns o (B, T, H, D), h_final and, with ``residuals``, the
    intermediates in the batch-major layout of the fused residuals."""
    if GATES != "activated":
        raise Gdn2ShapeError("raw gates need D = 64 or 128")
    q = torch.as_tensor(q)
    B, L, H, D, bt = _check_seq(q)
    Aqk, Akk = build_chunk_scores_pallas(q, k, b, g, scale)
    A = wy_solve_pallas(Akk)
    wp, u, kg, qg, gcl = recompute_wy_pallas(q, k, v, w, b, g, A)
    o, hf, hpre, vall = gdn2_inter_chunk_combine_with_state(Aqk, wp, u, kg, qg, gcl, scale, h0,
                                                            debug_tag)
    out = o.permute(0, 2, 3, 1, 4).reshape(B, L, H, D)
    res = None
    if residuals:
        res = dict(Aqk=Aqk, A=A, w_pseudo=wp, u=u, kg=kg, qg=qg, gc_last=gcl,
                   h_pre_all=hpre.permute(1, 2, 0, 3, 4), v_new_all=vall.permute(1, 2, 0, 3, 4),
                   Akk=Akk)
    return out, hf, res
