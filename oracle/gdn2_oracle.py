"""CPU oracle for the GDN-2 chunked forward and fused backward (float64 numpy).

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import this module, and only as the
checker or the timed CPU baseline; the library never calls it.

This is a restatement, stage by stage, of the reference algorithm
(Akseleu-J/gdn2-jax-kernel).  Each function cites the reference file:line it
follows.  Arrays are float64; the chunked layout is (B, H, nc, BT, ·).

Parity pin: ``tests/golden/*.npz`` hold outputs of the reference source itself
(executed in float64 on a numpy interpreter of the JAX calls it makes, see
``tests/golden/make_golden.py``) for N_SUB == 2, D == 128 — the cases the
reference computes correctly.  ``tests/test_oracle.py`` checks this module
against them, against the token-level recurrence and against float64 torch
autograd.

Deviations from the reference source, each the mathematically intended
behaviour:
  * ``wy_solve`` composes any number of BC sub-blocks with the same block
    recurrence that ``_block_solve`` uses for micro-blocks
    (gdn2_fwd.py:202-211); the reference hard-codes N_SUB == 2
    (gdn2_fwd.py:228-243) and leaves later rows zero otherwise.
  * h_pre_all / v_new_all are kept batch-major (B, H, nc, ·, ·), the layout
    every backward stage indexes (gdn2_bwd.py:104, 224); the reference's scan
    stacks them chunk-major (gdn2_fwd.py:393).
  * BT, BC, CLIP are arguments read at call time instead of module constants
    copied at import (gdn2_bwd.py:23, gdn2_pipeline.py:14-15).
  * D is not restricted to 128 (gdn2_fwd.py:145, gdn2_bwd.py:348).
"""
from __future__ import annotations

import numpy as np

MB = 16          # micro-block of the triangular solve, gdn2_fwd.py:32
FINAL_CLIP = 1e4  # gdn2_pipeline.py:34
PAIR_CLIP = 20.0  # exponent clip of pair decays, gdn2_fwd.py:125


def sanitize(x, clip):
    """clip to ±clip then nan→0, ±inf→±clip (gdn2_fwd.py:42-44)."""
    return np.nan_to_num(np.clip(x, -clip, clip), nan=0.0, posinf=clip, neginf=-clip)


def to_chunks(t, BT):
    """(B,T,H,D) → (B,H,nc,BT,D) (gdn2_fwd.py:79-82)."""
    B, T, H, D = t.shape
    return np.moveaxis(t.reshape(B, T // BT, BT, H, D), (1, 3), (2, 1))


def from_chunks(t):
    """(B,H,nc,BT,D) → (B,T,H,D) (gdn2_fwd.py:85-89)."""
    B, H, nc, BT, D = t.shape
    return np.moveaxis(t, (1, 2, 3), (3, 1, 2)).reshape(B, nc * BT, H, D)


def chunk_cumsum(g_r):
    """In-chunk inclusive cumulative sum of the log decay (gdn2_fwd.py:105-107)."""
    return np.cumsum(g_r, axis=-2)


# ----------------------------------------------------------------- forward
def chunk_scores(q, k, b, g, scale, BT, BC, clip):
    """Kernel A: Aqk, Akk per chunk (gdn2_fwd.py:99-139, 142-170).

    Aqk[i,j] = scale Σ_d q_id k_jd exp(clip(gc_id-gc_jd, ±20)), j ≤ i;
    Akk[i,j] = Σ_d b_id k_id k_jd exp(...), j < i; both sanitised.
    """
    q_r, k_r, b_r, g_r = (to_chunks(t, BT) for t in (q, k, b, g))
    gc = chunk_cumsum(g_r)
    lead = q_r.shape[:3]
    Aqk = np.zeros(lead + (BT, BT))
    Akk = np.zeros(lead + (BT, BT))
    bk = b_r * k_r
    n_sub = BT // BC
    idx = np.arange(BC)
    causal = (idx[:, None] >= idx[None, :]).astype(np.float64)
    strict = (idx[:, None] > idx[None, :]).astype(np.float64)
    for si in range(n_sub):
        for sj in range(si + 1):
            I = slice(si * BC, (si + 1) * BC)
            J = slice(sj * BC, (sj + 1) * BC)
            dd = gc[..., I, None, :] - gc[..., None, J, :]
            ed = np.exp(np.clip(dd, -PAIR_CLIP, PAIR_CLIP))
            aqk = scale * np.einsum("...id,...ijd,...jd->...ij", q_r[..., I, :], ed, k_r[..., J, :])
            akk = np.einsum("...id,...ijd,...jd->...ij", bk[..., I, :], ed, k_r[..., J, :])
            if si == sj:
                aqk = aqk * causal
                akk = akk * strict
            Aqk[..., I, J] = sanitize(aqk, clip)
            Akk[..., I, J] = sanitize(akk, clip)
    return Aqk, Akk


def _micro_solve(T, clip):
    """Row-by-row forward substitution of (I+T)^{-1}, T strictly lower MB×MB
    (gdn2_fwd.py:174-189)."""
    n = T.shape[-1]
    A = np.zeros(T.shape)
    eye = np.eye(n)
    for i in range(n):
        contrib = np.einsum("...r,...rc->...c", T[..., i, :], A)
        A[..., i, :] = sanitize(eye[i] - contrib, clip)
    return A


def _compose(T, n_blk, blk, clip, diag_solve):
    """Block forward substitution: A_mm = solve(T_mm);
    A_mn = -A_mm Σ_{k=n}^{m-1} T_mk A_kn with sanitising after every
    accumulation (gdn2_fwd.py:192-222)."""
    lead = T.shape[:-2]
    A = np.zeros(lead + (n_blk * blk, n_blk * blk))
    S = lambda m: slice(m * blk, (m + 1) * blk)
    for m in range(n_blk):
        A_mm = sanitize(diag_solve(T[..., S(m), S(m)]), clip)
        A[..., S(m), S(m)] = A_mm
        for n in range(m - 1, -1, -1):
            acc = np.zeros(lead + (blk, blk))
            for kk in range(n, m):
                acc = sanitize(acc + T[..., S(m), S(kk)] @ A[..., S(kk), S(n)], clip)
            A[..., S(m), S(n)] = sanitize(-(A_mm @ acc), clip)
    return A


def wy_solve(Akk, BT, BC, clip):
    """Kernel B: A = (I + Akk)^{-1} per chunk (gdn2_fwd.py:225-260), with the
    sub-block level generalised from N_SUB == 2 to any BT/BC."""
    mb = min(MB, BC)

    def block_solve(T):  # gdn2_fwd.py:192-222
        return _compose(T, BC // mb, mb, clip, lambda t: _micro_solve(t, clip))

    return _compose(Akk, BT // BC, BC, clip, block_solve)


def recompute_wy(q, k, v, w, b, g, A, BT, clip):
    """Kernel C: W = A(b⊙k⊙e^gc), U = A(w⊙v), kg, qg, gc_last
    (gdn2_fwd.py:264-295, 298-330)."""
    q_r, k_r, v_r, w_r, b_r, g_r = (to_chunks(t, BT) for t in (q, k, v, w, b, g))
    gc = chunk_cumsum(g_r)
    kb_dec = b_r * k_r * np.exp(gc)
    W = sanitize(A @ kb_dec, clip)
    U = sanitize(A @ (w_r * v_r), clip)
    gc_last = gc[..., BT - 1, :]
    kg = sanitize(k_r * np.exp(gc_last[..., None, :] - gc), clip)
    qg = sanitize(q_r * np.exp(gc), clip)
    return W, U, kg, qg, sanitize(gc_last, clip)


def inter_chunk(Aqk, W, U, kg, qg, gc_last, scale, h0, clip):
    """Kernel D with state (gdn2_fwd.py:369-397): serial over chunks,
    vnew = U - W h; o = scale qg h + Aqk vnew; h ← e^{gc_last} ⊙ h + kgᵀ vnew.
    Returns o (B,H,nc,BT,D), h_final, h_pre_all and v_new_all (batch-major)."""
    B, H, nc, BT, D = W.shape
    h = sanitize(h0, clip)  # gdn2_fwd.py:334-335
    o = np.zeros(W.shape)
    h_pre = np.zeros((B, H, nc, D, D))
    v_new = np.zeros(W.shape)
    for c in range(nc):
        h_pre[:, :, c] = h
        vn = U[:, :, c] - W[:, :, c] @ h
        oc = scale * (qg[:, :, c] @ h) + Aqk[:, :, c] @ vn
        h = sanitize(h * np.exp(gc_last[:, :, c])[..., None] + np.swapaxes(kg[:, :, c], -1, -2) @ vn, clip)
        o[:, :, c] = sanitize(oc, clip)
        v_new[:, :, c] = vn
    return o, h, h_pre, v_new


def forward(q, k, v, w, b, g, scale, h0=None, BT=64, BC=16, clip=1e4, residuals=False):
    """gdn2_pallas_forward (gdn2_fwd.py:400-424): A → B → C → D."""
    B, T, H, D = q.shape
    f = lambda t: np.asarray(t, dtype=np.float64)
    q, k, v, w, b, g = map(f, (q, k, v, w, b, g))
    h0 = np.zeros((B, H, D, D)) if h0 is None else f(h0)
    Aqk, Akk = chunk_scores(q, k, b, g, scale, BT, BC, clip)
    A = wy_solve(Akk, BT, BC, clip)
    W, U, kg, qg, gc_last = recompute_wy(q, k, v, w, b, g, A, BT, clip)
    o, h_final, h_pre, v_new = inter_chunk(Aqk, W, U, kg, qg, gc_last, scale, h0, clip)
    out = from_chunks(o)
    if residuals:
        return out, h_final, dict(Aqk=Aqk, Akk=Akk, A=A, W=W, U=U, kg=kg, qg=qg,
                                  gc_last=gc_last, h_pre=h_pre, v_new=v_new)
    return out, h_final


# ---------------------------------------------------------------- backward
def reverse_cumsum(dgc, clip):
    """B5: dg_i = Σ_{j≥i} dgc_j within a chunk (gdn2_bwd.py:32-41)."""
    return sanitize(np.flip(np.cumsum(np.flip(dgc, -2), axis=-2), -2), clip)


def dhu_backward(do_r, dv_partial, W, qg, kg, gc_last, scale, dht, clip):
    """B1: reverse scan over chunks (gdn2_bwd.py:45-80).
    dv_new = dv_partial + kg dh; dh_pre = qgᵀ(scale do) + e^{gc_last}⊙dh - Wᵀ dv_new."""
    B, H, nc, BT, D = W.shape
    dh = sanitize(dht, clip)
    dh_all = np.zeros((B, H, nc, D, D))
    dv_all = np.zeros(W.shape)
    T = lambda x: np.swapaxes(x, -1, -2)
    for c in range(nc - 1, -1, -1):
        dvn = sanitize(dv_partial[:, :, c] + kg[:, :, c] @ dh, clip)
        dhp = (T(qg[:, :, c]) @ (scale * do_r[:, :, c])
               + dh * np.exp(gc_last[:, :, c])[..., None] - T(W[:, :, c]) @ dvn)
        dh = sanitize(dhp, clip)
        dh_all[:, :, c] = dh
        dv_all[:, :, c] = dvn
    return dh_all, dh, dv_all


def dav_backward(Aqk, v_new, do_r, clip):
    """B2: dAqk = (do v_newᵀ)⊙causal, dv_partial = Aqkᵀ do (gdn2_bwd.py:84-122)."""
    BT = Aqk.shape[-1]
    causal = np.tril(np.ones((BT, BT)))
    dAqk = (do_r @ np.swapaxes(v_new, -1, -2)) * causal
    dv = np.swapaxes(Aqk, -1, -2) @ do_r
    return sanitize(dAqk, clip), sanitize(dv, clip)


def wy_dqkg_backward(q_r, k_r, b_r, w_r, v_r, gc, A, h_pre, v_new, do_r, dv, dh_next, scale, clip):
    """B3: gradients through W, U, A^{-1}, kg, qg, e^{gc} and the state decay
    (gdn2_bwd.py:126-210)."""
    BT = q_r.shape[-2]
    T = lambda x: np.swapaxes(x, -1, -2)
    gc_last = gc[..., BT - 1, :]
    eg = np.exp(gc)
    kb_dec = b_r * k_r * eg
    kg = k_r * np.exp(gc_last[..., None, :] - gc)
    qg = q_r * eg
    wv = w_r * v_r
    dqg = (scale * do_r) @ T(h_pre)
    dWp = (-dv) @ T(h_pre)
    dkg = v_new @ T(dh_next)
    dA = sanitize(dWp @ T(kb_dec) + dv @ T(wv), clip)
    dkb = T(A) @ dWp
    dwv = T(A) @ dv
    strict = np.tril(np.ones((BT, BT)), -1)
    tmp = sanitize(dA @ T(A), clip)
    dAkk = -(T(A) @ tmp) * strict
    dk = dkb * eg * b_r + dkg * np.exp(gc_last[..., None, :] - gc)
    db = dkb * eg * k_r
    dx = dkg * kg
    dgc = dkb * kb_dec + dqg * qg - dx
    dq = dqg * eg
    dw = dwv * v_r
    dv_raw = dwv * w_r
    dgc_last = dx.sum(-2) + np.exp(gc_last) * np.sum(dh_next * h_pre, axis=-1)
    dgc[..., BT - 1, :] += dgc_last
    s = lambda x: sanitize(x, clip)
    return dict(dq=s(dq), dk=s(dk), db=s(db), dw=s(dw), dv_raw=s(dv_raw),
                dgc=s(dgc), dAkk=s(dAkk))


def intra_backward(dAqk, dAkk, q, k, b, g, scale, BT, BC, clip):
    """B4: backward of Kernel A per sub-block pair, with the ±20 clip mask on
    the decay derivative and clipped accumulation (gdn2_bwd.py:248-339)."""
    q_r, k_r, b_r, g_r = (to_chunks(t, BT) for t in (q, k, b, g))
    gc = chunk_cumsum(g_r)
    bk = b_r * k_r
    dq = np.zeros(q_r.shape)
    dk = np.zeros(q_r.shape)
    dbk = np.zeros(q_r.shape)
    dgc = np.zeros(q_r.shape)
    idx = np.arange(BC)
    causal = (idx[:, None] >= idx[None, :]).astype(np.float64)
    strict = (idx[:, None] > idx[None, :]).astype(np.float64)
    acc = lambda x: sanitize(x, clip)
    for si in range(BT // BC):
        for sj in range(si + 1):
            I = slice(si * BC, (si + 1) * BC)
            J = slice(sj * BC, (sj + 1) * BC)
            dd = gc[..., I, None, :] - gc[..., None, J, :]
            cm = ((dd >= -PAIR_CLIP) & (dd <= PAIR_CLIP)).astype(np.float64)
            ed = np.exp(np.clip(dd, -PAIR_CLIP, PAIR_CLIP))
            dMq = dAqk[..., I, J]
            dMk = dAkk[..., I, J]
            if si == sj:
                dMq = dMq * causal
                dMk = dMk * strict
            Lq = scale * q_r[..., I, :]
            Lk = bk[..., I, :]
            R = k_r[..., J, :]
            dLq = np.einsum("...ij,...ijd,...jd->...id", dMq, ed, R)
            dRq = np.einsum("...ij,...ijd,...id->...jd", dMq, ed, Lq)
            wq = dMq[..., None] * Lq[..., :, None, :] * R[..., None, :, :] * ed * cm
            dLk = np.einsum("...ij,...ijd,...jd->...id", dMk, ed, R)
            dRk = np.einsum("...ij,...ijd,...id->...jd", dMk, ed, Lk)
            wk = dMk[..., None] * Lk[..., :, None, :] * R[..., None, :, :] * ed * cm
            dq[..., I, :] = acc(dq[..., I, :] + dLq * scale)
            dbk[..., I, :] = acc(dbk[..., I, :] + dLk)
            dk[..., J, :] = acc(dk[..., J, :] + dRq + dRk)
            dgc[..., I, :] = acc(dgc[..., I, :] + wq.sum(-2) + wk.sum(-2))
            dgc[..., J, :] = acc(dgc[..., J, :] - wq.sum(-3) - wk.sum(-3))
    s = lambda x: sanitize(x, clip)
    return s(dq), s(dk + dbk * b_r), s(dbk * k_r), s(dgc)


def backward(q, k, v, w, b, g, scale, h0, dout, dh_final, BT=64, BC=16, clip=1e4):
    """Fused backward of the custom_vjp (gdn2_pipeline.py:70-137): recompute the
    forward, then B2 → B1 → B3 → B4 → B5, sum, final ±1e4 sanitise.
    Returns (dq, dk, dv, dw, db, dg, dh0) in float64."""
    f = lambda t: np.asarray(t, dtype=np.float64)
    q, k, v, w, b, g, dout, dh_final = map(f, (q, k, v, w, b, g, dout, dh_final))
    B, T, H, D = q.shape
    h0 = np.zeros((B, H, D, D)) if h0 is None else f(h0)
    _, _, r = forward(q, k, v, w, b, g, scale, h0, BT, BC, clip, residuals=True)
    gc = chunk_cumsum(to_chunks(g, BT))
    q_r, k_r, b_r, w_r, v_r, do_r = (to_chunks(t, BT) for t in (q, k, b, w, v, dout))
    dAqk, dv_partial = dav_backward(r["Aqk"], r["v_new"], do_r, clip)
    dh_all, dh0, dv_all = dhu_backward(do_r, dv_partial, r["W"], r["qg"], r["kg"],
                                       r["gc_last"], scale, dh_final, clip)
    dh_next = np.concatenate([dh_all[:, :, 1:], dh_final[:, :, None]], axis=2)  # gdn2_pipeline.py:52-56
    b3 = wy_dqkg_backward(q_r, k_r, b_r, w_r, v_r, gc, r["A"], r["h_pre"], r["v_new"],
                          do_r, dv_all, dh_next, scale, clip)
    dq4, dk4, db4, dgc4 = intra_backward(dAqk, b3["dAkk"], q, k, b, g, scale, BT, BC, clip)
    dg = reverse_cumsum(b3["dgc"] + dgc4, clip)
    fs = lambda x: sanitize(x, FINAL_CLIP)
    return (fs(from_chunks(b3["dq"] + dq4)), fs(from_chunks(b3["dk"] + dk4)),
            fs(from_chunks(b3["dv_raw"])), fs(from_chunks(b3["dw"])),
            fs(from_chunks(b3["db"] + db4)), fs(from_chunks(dg)), fs(dh0))


# ------------------------------------------------- independent restatement
def token_recurrence(q, k, v, w, b, g, scale, h0=None):
    """Token-level form of the same model (no chunking, no clips):
    S̃ = e^{g_t} ⊙ S (row scaling); vnew = w⊙v - (b⊙k)ᵀ S̃; S = S̃ + k ⊗ vnew;
    o = scale qᵀ S.  Equal to the chunked form up to the ±20 pair clip."""
    f = lambda t: np.asarray(t, dtype=np.float64)
    q, k, v, w, b, g = map(f, (q, k, v, w, b, g))
    B, T, H, D = q.shape
    S = np.zeros((B, H, D, D)) if h0 is None else f(h0).copy()
    o = np.zeros(q.shape)
    for t in range(T):
        S = S * np.exp(g[:, t])[..., None]
        vn = w[:, t] * v[:, t] - np.einsum("bhd,bhdv->bhv", b[:, t] * k[:, t], S)
        S = S + k[:, t][..., None] * vn[..., None, :]
        o[:, t] = scale * np.einsum("bhd,bhdv->bhv", q[:, t], S)
    return o, S


def gdn2_chunked_wy_reference(q, k, v, g, b, w, scale, chunk_size=64, h0=None, BC=None, clip=1e4):
    """Entry point named by the reference's tests (tests/test_reference.py:4, 19);
    note the argument order g, b, w."""
    BC = BC or min(chunk_size, 64)
    return forward(q, k, v, w, b, g, scale, h0, chunk_size, BC, clip)
