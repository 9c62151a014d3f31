"""The reference's stage functions (gdn2_fwd.py:142-397, gdn2_bwd.py:32-375)
as separate CUDA entry points, each against the float64 oracle's stage on
the same inputs, and the reference's backward pipeline composed from them
(gdn2_pipeline.py:70-137) against the fused backward.  Tolerance rel-L2 1e-4.
"""
import numpy as np
import pytest
import torch

import gdn2_oracle as O
from conftest import cuda_ok
from gdn2_package import gdn2_backward, gdn2_bwd, gdn2_fwd
from gdn2_package.synthetic import make_inputs

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

NAMES = ("q", "k", "v", "w", "b", "g")
CASES = [(64, 16, 1e4), (128, 64, 1e4), (64, 32, 0.5),   # BT, BC, CLIP (0.5: clips act)
         (256, 128, 1e4), (256, 64, 0.5)]                  # BT = 256: the reference's default


def rel(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / max(float(b.norm()), 1e-300))


def _setup(BT, BC, clip, seed=3):
    gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = BT, BC, clip
    inp = make_inputs(2, 256, 2, 128, seed=seed, h0_std=0.1)
    x = {n: inp[n].astype(np.float64) for n in NAMES}
    return inp, x


def _cu(a):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float32).cuda()


@pytest.mark.parametrize("BT,BC,clip", CASES)
def test_forward_stages_vs_oracle(BT, BC, clip):
    inp, x = _setup(BT, BC, clip)
    s = inp["scale"]
    dev = {n: _cu(inp[n]) for n in NAMES}
    Aqk, Akk = gdn2_fwd.build_chunk_scores_pallas(dev["q"], dev["k"], dev["b"], dev["g"], s)
    Aqk_r, Akk_r = O.chunk_scores(x["q"], x["k"], x["b"], x["g"], s, BT, BC, clip)
    assert rel(Aqk, Aqk_r) < 1e-4 and rel(Akk, Akk_r) < 1e-4, (rel(Aqk, Aqk_r), rel(Akk, Akk_r))
    A = gdn2_fwd.wy_solve_pallas(_cu(Akk_r))
    A_r = O.wy_solve(Akk_r, BT, BC, clip)
    assert rel(A, A_r) < 1e-4, rel(A, A_r)
    outs = gdn2_fwd.recompute_wy_pallas(*[dev[n] for n in NAMES], _cu(A_r))
    refs = O.recompute_wy(*[x[n] for n in NAMES], A_r, BT, clip)
    for name, a, r in zip(("w_pseudo", "u", "kg", "qg", "gc_last"), outs, refs):
        assert rel(a, r) < 1e-4, (name, rel(a, r))
    W, U, kg, qg, gcl = refs
    o, hf, hpre, vall = gdn2_fwd.gdn2_inter_chunk_combine_with_state(
        _cu(Aqk_r), _cu(W), _cu(U), _cu(kg), _cu(qg), _cu(gcl), s, _cu(inp["h0"]))
    o_r, h_r, hpre_r, vn_r = O.inter_chunk(Aqk_r, W, U, kg, qg, gcl, s, inp["h0"], clip)
    assert rel(o, o_r) < 1e-4 and rel(hf, h_r) < 1e-4, (rel(o, o_r), rel(hf, h_r))
    # the reference's scan stacks the residuals chunk-major
    assert rel(hpre.permute(1, 2, 0, 3, 4), hpre_r) < 1e-4
    assert rel(vall.permute(1, 2, 0, 3, 4), vn_r) < 1e-4
    o2, h2 = gdn2_fwd.gdn2_inter_chunk_combine(_cu(Aqk_r), _cu(W), _cu(U), _cu(kg), _cu(qg),
                                               _cu(gcl), s, _cu(inp["h0"]))
    assert torch.equal(o2, o) and torch.equal(h2, hf)


@pytest.mark.parametrize("BT,BC,clip", CASES)
def test_backward_stages_vs_oracle(BT, BC, clip):
    inp, x = _setup(BT, BC, clip, seed=4)
    s = inp["scale"]
    _, _, res = O.forward(*[x[n] for n in NAMES], s, inp["h0"], BT, BC, clip, residuals=True)
    do_r = O.to_chunks(inp["dout"].astype(np.float64), BT)
    # B2
    dAqk, dvp = gdn2_bwd.dav_backward_pallas(_cu(res["Aqk"]), _cu(res["v_new"]), _cu(do_r))
    dAqk_r, dvp_r = O.dav_backward(res["Aqk"], res["v_new"], do_r, clip)
    assert rel(dAqk, dAqk_r) < 1e-4 and rel(dvp, dvp_r) < 1e-4
    # B1
    dh_all, dh0, dv_all = gdn2_bwd.gdn2_dhu_backward(
        _cu(do_r), _cu(dvp_r), _cu(res["W"]), _cu(res["qg"]), _cu(res["kg"]), _cu(res["gc_last"]),
        s, _cu(inp["dh_final"]))
    dh_all_r, dh0_r, dv_all_r = O.dhu_backward(do_r, dvp_r, res["W"], res["qg"], res["kg"],
                                               res["gc_last"], s, inp["dh_final"], clip)
    for name, a, r in (("dh_all", dh_all, dh_all_r), ("dh0", dh0, dh0_r), ("dv_all", dv_all, dv_all_r)):
        assert rel(a, r) < 1e-4, (name, rel(a, r))
    # B3
    ch = lambda n: O.to_chunks(x[n], BT)
    gc = O.chunk_cumsum(ch("g"))
    dh_next = np.concatenate([dh_all_r[:, :, 1:], inp["dh_final"][:, :, None].astype(np.float64)], 2)
    b3 = gdn2_bwd.wy_dqkg_backward_pallas(
        *[_cu(ch(n)) for n in ("q", "k", "b", "w", "v")], _cu(gc), _cu(res["A"]), None,
        _cu(res["h_pre"]), _cu(res["v_new"]), _cu(do_r), _cu(dv_all_r), _cu(dh_next), s)
    b3_r = O.wy_dqkg_backward(ch("q"), ch("k"), ch("b"), ch("w"), ch("v"), gc, res["A"],
                              res["h_pre"], res["v_new"], do_r, dv_all_r, dh_next, s, clip)
    for name in ("dq", "dk", "db", "dw", "dv_raw", "dgc", "dAkk"):
        assert rel(b3[name], b3_r[name]) < 1e-4, (name, rel(b3[name], b3_r[name]))
    # B4
    dq4, dk4, db4, dgc4 = gdn2_bwd.intra_backward_pallas(
        _cu(dAqk_r), _cu(b3_r["dAkk"]), *[_cu(inp[n]) for n in ("q", "k", "b", "g")], s)
    r4 = O.intra_backward(dAqk_r, b3_r["dAkk"], x["q"], x["k"], x["b"], x["g"], s, BT, BC, clip)
    for name, a, r in zip(("dq", "dk", "db", "dgc"), (dq4, dk4, db4, dgc4), r4):
        assert rel(a, r) < 1e-4, (name, rel(a, r))
    # B5
    dgc_tot = b3_r["dgc"] + r4[3]
    dg = gdn2_bwd.reverse_cumsum_bwd(_cu(dgc_tot), BT)
    assert rel(dg, O.reverse_cumsum(dgc_tot, clip)) < 1e-4


@pytest.mark.parametrize("BT,BC", [(64, 16), (128, 64), (256, 128)])
def test_reference_pipeline_from_stages(BT, BC):
    """_gdn2_core_bwd (gdn2_pipeline.py:70-137) written with the stage
    functions gives the fused backward's gradients."""
    inp, _ = _setup(BT, BC, 1e4, seed=6)
    s = inp["scale"]
    q, k, v, w, b, g = (_cu(inp[n]) for n in NAMES)
    h0, do, dhf = _cu(inp["h0"]), _cu(inp["dout"]), _cu(inp["dh_final"])
    B, L, H, D = q.shape
    nc = L // BT
    F, Bw = gdn2_fwd, gdn2_bwd
    Aqk, Akk = F.build_chunk_scores_pallas(q, k, b, g, s)
    A = F.wy_solve_pallas(Akk)
    wp, u, kg, qg, gcl = F.recompute_wy_pallas(q, k, v, w, b, g, A)
    _, _, hpre, vall = F.gdn2_inter_chunk_combine_with_state(Aqk, wp, u, kg, qg, gcl, s, h0=h0)
    hpre, vall = hpre.permute(1, 2, 0, 3, 4), vall.permute(1, 2, 0, 3, 4)   # to batch-major
    ch = lambda t: t.reshape(B, nc, BT, H, D).permute(0, 3, 1, 2, 4).contiguous()
    gc = torch.cumsum(ch(g), dim=-2)
    dAqk, dvp = Bw.dav_backward_pallas(Aqk, vall, ch(do))
    dh_all, dh0, dv_all = Bw.gdn2_dhu_backward(ch(do), dvp, wp, qg, kg, gcl, s, dht=dhf)
    dh_next = torch.cat([dh_all[:, :, 1:], dhf[:, :, None]], dim=2)
    b3 = Bw.wy_dqkg_backward_pallas(ch(q), ch(k), ch(b), ch(w), ch(v), gc, A, Akk, hpre, vall,
                                    ch(do), dv_all, dh_next, s)
    dq4, dk4, db4, dgc4 = Bw.intra_backward_pallas(dAqk, b3["dAkk"], q, k, b, g, s)
    dg = Bw.reverse_cumsum_bwd(b3["dgc"] + dgc4, BT)
    unch = lambda t: t.permute(0, 2, 3, 1, 4).reshape(B, L, H, D)
    fin = lambda t: torch.nan_to_num(t.clamp(-1e4, 1e4), nan=0.0, posinf=1e4, neginf=-1e4)
    staged = [fin(unch(t)) for t in (b3["dq"] + dq4, b3["dk"] + dk4, b3["dv_raw"], b3["dw"],
                                     b3["db"] + db4, dg)] + [fin(dh0)]
    fused = gdn2_backward(q, k, v, w, b, g, s, h0, do, dhf)
    for name, a, r in zip(("dq", "dk", "dv", "dw", "db", "dg", "dh0"), staged, fused):
        assert rel(a, r) < 1e-4, (name, rel(a, r))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("BT,BC,clip", [(64, 16, 1e4), (128, 64, 1e4), (64, 32, 0.5)])
def test_head_dim_256_vs_oracle(BT, BC, clip, dtype):
    """D = 256 (beyond the reference's D = 128) runs the reference's own
    stage composition on the stage kernels: forward, all seven gradients and
    the autograd path against the float64 oracle."""
    from gdn2_package import gdn2_pallas_forward, gdn2_pallas_forward_trainable
    gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = BT, BC, clip
    inp = make_inputs(1, 256, 2, 256, seed=12, h0_std=0.1)
    args = [torch.as_tensor(inp[n]).to("cuda", dtype) for n in NAMES]
    h0 = _cu(inp["h0"])
    ref_in = [torch.as_tensor(inp[n]).to(dtype).double().numpy() for n in NAMES]
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    o, h = gdn2_pallas_forward(*args, inp["scale"], h0)
    o_r, h_r = O.forward(*ref_in, inp["scale"], inp["h0"], BT, BC, clip)
    assert rel(o, o_r) < tol and rel(h, h_r) < tol, (rel(o, o_r), rel(h, h_r))
    grads = gdn2_backward(*args, inp["scale"], h0, _cu(inp["dout"]), _cu(inp["dh_final"]))
    g_r = O.backward(*ref_in, inp["scale"], inp["h0"], inp["dout"], inp["dh_final"], BT, BC, clip)
    for name, a, r in zip(("dq", "dk", "dv", "dw", "db", "dg", "dh0"), grads, g_r):
        assert rel(a, r) < tol, (name, rel(a, r))
    xs = [a.clone().requires_grad_() for a in args]
    h0g = h0.clone().requires_grad_()
    o2, h2 = gdn2_pallas_forward_trainable(*xs, inp["scale"], h0g)
    torch.autograd.backward((o2, h2), (_cu(inp["dout"]), _cu(inp["dh_final"])))
    assert torch.equal(o2.detach(), o)
    for a, b in zip([*(x.grad for x in xs), h0g.grad], grads):
        assert torch.equal(a, b)


def test_head_dim_256_shape_limits():
    from gdn2_package import gdn2_pallas_forward
    gdn2_fwd.BT, gdn2_fwd.BC = 256, 128
    x = torch.zeros((1, 256, 1, 256), device="cuda")
    with pytest.raises(gdn2_fwd.Gdn2ShapeError):
        gdn2_pallas_forward(x, x, x, x, x, x, 0.06)
