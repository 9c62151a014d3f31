"""Token-by-token decode with a carried state (no counterpart in the reference).

``gdn2_decode(q, k, v, w, b, g, scale, h0=None)`` runs a short segment
(B, T, H, D) token by token from the state ``h0`` (B, H, D, D) and returns
``(o, h_final)`` like ``gdn2_pallas_forward`` (gdn2_fwd.py:400-404).  It is
the chunked forward with chunks of one token: the same recurrence, with the
module's ``CLIP`` sanitiser after every token.  Any T works, but the cost is
linear in T with no chunk parallelism, so prompts belong to
``gdn2_pallas_forward`` and per-step generation to this function.
"""
from __future__ import annotations

import torch

from . import _lib
from . import gdn2_fwd as _fwd


def gdn2_decode(q, k, v, w, b, g, scale, h0=None):
    ts = tuple(torch.as_tensor(t) for t in (q, k, v, w, b, g))
    shape = tuple(ts[0].shape)
    if len(shape) != 4 or any(tuple(t.shape) != shape for t in ts):
        raise _fwd.Gdn2ShapeError(f"inputs must share one (B, T, H, D) shape; got {shape}")
    B, T, H, D = shape
    if D not in (64, 128):
        raise _fwd.Gdn2ShapeError(f"head dim D={D} unsupported (64 or 128)")
    if B * T * H == 0:
        raise _fwd.Gdn2ShapeError("empty problem")
    on_host = ts[0].device.type != "cuda"
    dev = torch.device("cuda", torch.cuda.current_device()) if on_host else ts[0].device
    cdt = torch.bfloat16 if all(t.dtype == torch.bfloat16 for t in ts) else torch.float32
    x = [t.to(device=dev, dtype=cdt, non_blocking=True).contiguous() for t in ts]
    hs = None
    if h0 is not None:
        hs = torch.as_tensor(h0).to(device=dev, dtype=torch.float32, non_blocking=True).contiguous()
        if tuple(hs.shape) != (B, H, D, D):
            raise _fwd.Gdn2ShapeError(f"h0 must be {(B, H, D, D)}; got {tuple(hs.shape)}")
    o = torch.empty((B, T, H, D), dtype=torch.float32, device=dev)
    hf = torch.empty((B, H, D, D), dtype=torch.float32, device=dev)
    code = _lib.F32 if cdt == torch.float32 else _lib.BF16
    if _fwd.GATES == "raw":
        code |= _lib.GATES_RAW
    rc = _lib.load().gdn2_decode(code,
                                 *[t.data_ptr() for t in x],
                                 hs.data_ptr() if hs is not None else None, o.data_ptr(),
                                 hf.data_ptr(), B, T, H, D, float(scale), float(_fwd.CLIP),
                                 torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(rc, "gdn2_decode")
    if on_host:
        return o.cpu(), hf.cpu()
    return o, hf
