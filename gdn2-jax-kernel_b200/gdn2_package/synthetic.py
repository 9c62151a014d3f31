"""Seeded synthetic GDN-2 inputs with the benchmark's distributions.

Draw order and distributions (one ``numpy.random.default_rng(seed)`` stream):
q, k ~ N(0,1) then L2-normalised over D per (b, t, h); v ~ N(0,1);
w, b = sigmoid(N(0,1)); g = -softplus(N(0,1)); h0 ~ N(0, h0_std) when
requested; dout ~ N(0,1); dh_final ~ N(0,1).  ``scale = 1/sqrt(D)``.
"""
from __future__ import annotations

import numpy as np


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _softplus(x):
    return np.log1p(np.exp(-np.abs(x))) + np.maximum(x, 0.0)


def make_inputs(B, T, H, D, seed=0, h0_std=None, grads=True, dtype=np.float32):
    """Return a dict of numpy arrays: q k v w b g [h0] [dout dh_final], scale."""
    rng = np.random.default_rng(seed)
    shape = (B, T, H, D)

    def nrm(s):
        return rng.standard_normal(s, dtype=np.float64)

    q = nrm(shape)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k = nrm(shape)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = nrm(shape)
    w = _sigmoid(nrm(shape))
    b = _sigmoid(nrm(shape))
    g = -_softplus(nrm(shape))
    out = dict(q=q, k=k, v=v, w=w, b=b, g=g)
    if h0_std is not None:
        out["h0"] = h0_std * nrm((B, H, D, D))
    if grads:
        out["dout"] = nrm(shape)
        out["dh_final"] = nrm((B, H, D, D))
    out = {n: a.astype(dtype) for n, a in out.items()}
    out["scale"] = float(1.0 / np.sqrt(D))
    return out


def make_inputs_torch(B, T, H, D, seed=0, device="cuda", h0_std=None, grads=True):
    """The same distributions drawn by torch on ``device`` (float32), for
    benchmark sizes whose host-side generation would take minutes.  The values
    are not bit-identical to ``make_inputs``."""
    import torch

    gen = torch.Generator(device=device).manual_seed(seed)
    shape = (B, T, H, D)

    def nrm(s):
        return torch.randn(s, generator=gen, device=device, dtype=torch.float32)

    q = torch.nn.functional.normalize(nrm(shape), dim=-1)
    k = torch.nn.functional.normalize(nrm(shape), dim=-1)
    out = dict(q=q, k=k, v=nrm(shape), w=torch.sigmoid(nrm(shape)), b=torch.sigmoid(nrm(shape)),
               g=-torch.nn.functional.softplus(nrm(shape)))
    if h0_std is not None:
        out["h0"] = h0_std * nrm((B, H, D, D))
    if grads:
        out["dout"] = nrm(shape)
        out["dh_final"] = nrm((B, H, D, D))
    out["scale"] = float(D ** -0.5)
    return out
