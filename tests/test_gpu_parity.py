"""Parity of the CUDA path (libgdn2.so through the package API) with the
float64 oracle and, at the benchmark sizes, with float64 torch autograd.

Tolerances (rel-L2, from the benchmark spec): 1e-4 for float32 inputs,
2e-2 for bfloat16 inputs (the reference is evaluated on the bf16-rounded
inputs).
"""
import os

import numpy as np
import pytest
import torch

import gdn2_oracle as O
import torch_ref
from conftest import cuda_ok
from gdn2_package import (gdn2_backward, gdn2_fwd, gdn2_pallas_forward,
                          gdn2_pallas_forward_trainable, gdn2_pallas_forward_with_residuals)
from gdn2_package.synthetic import make_inputs

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

NAMES = ("q", "k", "v", "w", "b", "g")
GRADS = ("dq", "dk", "dv", "dw", "db", "dg", "dh0")
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def rel(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / max(float(b.norm()), 1e-300))


def _set_consts(BT, BC, clip):
    gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = BT, BC, clip


def _dev(inp, dtype):
    return [torch.as_tensor(inp[n]).to("cuda", dtype) for n in NAMES]


def _rounded(inp, dtype):
    """Inputs as the kernel sees them (bf16-rounded), in float64 numpy."""
    return [torch.as_tensor(inp[n]).to(dtype).double().numpy() for n in NAMES]


SMALL = [  # B, T, H, D, BT, BC, h0_std
    (1, 256, 2, 64, 64, 16, None),      # benchmark config 0
    (2, 256, 2, 128, 128, 64, 0.1),
    (1, 384, 3, 128, 64, 16, 0.1),
    (2, 256, 2, 64, 128, 64, None),
    (1, 128, 2, 128, 128, 32, 0.1),     # a single chunk
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,T,H,D,BT,BC,h0s", SMALL)
def test_forward_backward_vs_oracle(B, T, H, D, BT, BC, h0s, dtype):
    _set_consts(BT, BC, 1e4)
    inp = make_inputs(B, T, H, D, seed=11, h0_std=h0s)
    h0 = torch.as_tensor(inp["h0"]).cuda() if "h0" in inp else None
    args = _dev(inp, dtype)
    o, h = gdn2_pallas_forward(*args, inp["scale"], h0)
    assert o.dtype == torch.float32 and h.dtype == torch.float32
    ref_in = _rounded(inp, dtype)
    o_r, h_r = O.forward(*ref_in, inp["scale"], inp.get("h0"), BT, BC, 1e4)
    tol = TOL[dtype]
    assert rel(o, o_r) < tol and rel(h, h_r) < tol, (rel(o, o_r), rel(h, h_r))
    grads = gdn2_backward(*args, inp["scale"], h0, torch.as_tensor(inp["dout"]).cuda(),
                          torch.as_tensor(inp["dh_final"]).cuda())
    g_r = O.backward(*ref_in, inp["scale"], inp.get("h0"), inp["dout"], inp["dh_final"], BT, BC, 1e4)
    for name, a, b in zip(GRADS, grads, g_r):
        if name != "dh0":
            assert a.dtype == dtype, name
        assert rel(a, b) < tol, (name, rel(a, b))


@pytest.mark.parametrize("exact", [False, True])
def test_bt64_chunking_policy(exact):
    """BT=64 with D=128: by default the kernels run 128-row chunks (tensor
    cores); EXACT_BT runs 64-row chunks (CUDA cores).  Both match the oracle
    run at BT=64, and each other to float32 rounding."""
    from gdn2_package import gdn2_fwd
    _set_consts(64, 16, 1e4)
    gdn2_fwd.EXACT_BT = exact
    inp = make_inputs(2, 512, 2, 128, seed=21, h0_std=0.1)
    args = _dev(inp, torch.float32)
    h0 = torch.as_tensor(inp["h0"]).cuda()
    o, h = gdn2_pallas_forward(*args, inp["scale"], h0)
    ref_in = _rounded(inp, torch.float32)
    o_r, h_r = O.forward(*ref_in, inp["scale"], inp["h0"], 64, 16, 1e4)
    assert rel(o, o_r) < 1e-5 and rel(h, h_r) < 1e-5, (rel(o, o_r), rel(h, h_r))
    grads = gdn2_backward(*args, inp["scale"], h0, torch.as_tensor(inp["dout"]).cuda(),
                          torch.as_tensor(inp["dh_final"]).cuda())
    g_r = O.backward(*ref_in, inp["scale"], inp["h0"], inp["dout"], inp["dh_final"], 64, 16, 1e4)
    for name, a, b in zip(GRADS, grads, g_r):
        assert rel(a, b) < 1e-5, (name, rel(a, b))


@pytest.mark.parametrize("D,BT,BC", [(128, 64, 16), (128, 128, 64), (64, 64, 16)])
def test_masked_tail(D, BT, BC):
    """T not a multiple of BT with MASKED_TAIL: the forward matches the float64
    token recurrence, the gradients match the oracle's backward on explicitly
    zero-padded inputs, restricted to the real tokens; the default refuses."""
    from gdn2_package import gdn2_fwd
    _set_consts(BT, BC, 1e4)
    T = 200
    inp = make_inputs(2, T, 2, D, seed=41, h0_std=0.1)
    args = _dev(inp, torch.float32)
    h0 = torch.as_tensor(inp["h0"]).cuda()
    with pytest.raises(AssertionError):
        gdn2_pallas_forward(*args, inp["scale"], h0)
    gdn2_fwd.MASKED_TAIL = True
    o, h = gdn2_pallas_forward(*args, inp["scale"], h0)
    assert o.shape == (2, T, 2, D)
    o_r, h_r = O.token_recurrence(*[inp[n] for n in NAMES], inp["scale"], inp["h0"])
    assert rel(o, o_r) < 1e-5 and rel(h, h_r) < 1e-5, (rel(o, o_r), rel(h, h_r))
    do = torch.as_tensor(inp["dout"]).cuda()
    dhf = torch.as_tensor(inp["dh_final"]).cuda()
    grads = gdn2_backward(*args, inp["scale"], h0, do, dhf)
    Tp = -(-T // BT) * BT
    padz = lambda a: np.concatenate([a, np.zeros((a.shape[0], Tp - T) + a.shape[2:], a.dtype)], 1)
    g_r = O.backward(*[padz(inp[n]) for n in NAMES], inp["scale"], inp["h0"], padz(inp["dout"]),
                     inp["dh_final"], BT, BC, 1e4)
    for name, a, b in zip(GRADS, grads, g_r):
        b = b[:, :T] if name != "dh0" else b
        assert a.shape == b.shape and rel(a, b) < 1e-4, (name, rel(a, b))


@pytest.mark.parametrize("name", ["ref_bt64_bc32", "ref_bt128_bc64", "ref_clip_bt128_bc64"])
def test_against_reference_golden(name, monkeypatch):
    """Outputs of the reference source itself (tests/golden/make_golden.py).
    ref_clip_bt128_bc64 runs CLIP = 20 with dout, dh_final x 30, so that
    dv_new = san(dv_partial + kg dh) clips inside the backward state chain
    (gdn2_bwd.py:66-68): the tensor-core backward must flag those (b, h) and
    recompute them with the exact step."""
    from gdn2_package import _lib
    monkeypatch.setattr(_lib, "CHECK_STATUS", "always")
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    B, T, H, D, BT, BC = (int(x) for x in z["meta"])
    _set_consts(BT, BC, float(z["clip"]))
    args = [torch.as_tensor(z[n]).cuda() for n in NAMES]
    h0 = torch.as_tensor(z["h0"]).cuda()
    o, h = gdn2_pallas_forward(*args, float(z["scale"]), h0)
    assert rel(o, z["o"]) < 1e-4 and rel(h, z["h_final"]) < 1e-4
    grads = gdn2_backward(*args, float(z["scale"]), h0, torch.as_tensor(z["dout"]).cuda(),
                          torch.as_tensor(z["dh_final"]).cuda())
    if name == "ref_clip_bt128_bc64":
        assert _lib.LAST_STATUS & _lib.STATUS_EXACT_RECOMPUTE
    for gname, a in zip(GRADS, grads):
        assert rel(a, z[gname]) < 1e-4, (gname, rel(a, z[gname]))


@pytest.mark.parametrize("clip,dscale,h0s,gscale", [
    (20.0, 30.0, 0.1, 1.0),    # dv_new clips inside the backward chain, B4 accumulators clip
    (0.3, 1.0, 0.1, 1.0),      # U, W, kg, o and the backward clip
    (0.5, 1.0, 0.1, 0.01),     # slow gates: the forward state h itself clips
    (1e3, 1.0, None, 1.0),     # nothing clips: the fast paths run, no recompute
])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("BT,BC", [(128, 64), (64, 16)])
def test_backward_with_clip_active(BT, BC, clip, dscale, h0s, gscale, dtype, monkeypatch):
    """The CLIP sanitiser acting, against the float64 oracle: o, h_final and
    all seven gradients.  BT = D = 128 runs the tcgen05 kernels (affine chain
    with its guard, B4 guard), BT = 64 the CUDA-core kernels (B4 guard)."""
    from gdn2_package import _lib
    monkeypatch.setattr(_lib, "CHECK_STATUS", "always")
    _set_consts(BT, BC, clip)
    inp = make_inputs(2, 768, 2, 128, seed=31, h0_std=h0s)
    inp["g"] = inp["g"] * np.float32(gscale)
    inp["dout"] = inp["dout"] * np.float32(dscale)
    inp["dh_final"] = inp["dh_final"] * np.float32(dscale)
    args = _dev(inp, dtype)
    h0 = torch.as_tensor(inp["h0"]).cuda() if "h0" in inp else None
    o, h = gdn2_pallas_forward(*args, inp["scale"], h0)
    ref_in = _rounded(inp, dtype)
    o_r, h_r = O.forward(*ref_in, inp["scale"], inp.get("h0"), BT, BC, clip)
    tol = TOL[dtype]
    assert rel(o, o_r) < tol and rel(h, h_r) < tol, (rel(o, o_r), rel(h, h_r))
    grads = gdn2_backward(*args, inp["scale"], h0, torch.as_tensor(inp["dout"]).cuda(),
                          torch.as_tensor(inp["dh_final"]).cuda())
    if BT == 128:
        recomputed = bool(_lib.LAST_STATUS & _lib.STATUS_EXACT_RECOMPUTE)
        assert recomputed == (clip < 1e3), _lib.LAST_STATUS
    if clip >= 1e3:
        assert not _lib.LAST_STATUS & _lib.STATUS_B4_EXACT, _lib.LAST_STATUS
    g_r = O.backward(*ref_in, inp["scale"], inp.get("h0"), inp["dout"], inp["dh_final"], BT, BC,
                     clip)
    for name, a, b in zip(GRADS, grads, g_r):
        assert rel(a, b) < tol, (name, rel(a, b))


def test_wait_timeout_surfaces_and_context_survives(monkeypatch):
    """A kernel whose barrier wait runs out records it in the workspace status
    and returns; the Python layer raises Gdn2Error; the next call clears the
    word and the CUDA context keeps working."""
    from gdn2_package import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    ws = torch.empty(4096, dtype=torch.uint8, device="cuda")
    assert lib.gdn2_selftest_wait_timeout(ws.data_ptr(), ws.numel(), 256, stream) == 0
    assert _lib.workspace_status(ws, stream) == _lib.STATUS_WAIT_TIMEOUT
    monkeypatch.setattr(_lib, "CHECK_STATUS", "always")
    with pytest.raises(_lib.Gdn2Error, match="timed out"):
        _lib.check_status(ws, stream, "selftest", synced=False)
    # a real call on a workspace whose word was set starts from a clear word
    _set_consts(128, 64, 1e4)
    inp = make_inputs(1, 256, 1, 128, seed=2, grads=False)
    from gdn2_package.gdn2_fwd import _Prepared, _run_forward
    p = _Prepared(*_dev(inp, torch.float32), inp["scale"], None)
    big = p.workspace(False)
    assert lib.gdn2_selftest_wait_timeout(big.data_ptr(), big.numel(), 64, stream) == 0
    o, h, _ = _run_forward(p, ws=big)
    assert _lib.LAST_STATUS == 0
    assert torch.isfinite(o).all() and float((torch.ones(4, device="cuda") * 2).sum()) == 8.0


def test_against_reference_golden_saturated():
    """The reference tests' all-ones inputs (g = +1 takes the exact
    elementwise path with the +-20 exponent clip); everything saturates."""
    z = np.load(os.path.join(GOLDEN, "ref_ones_bt64_bc32.npz"))
    B, T, H, D, BT, BC = (int(x) for x in z["meta"])
    _set_consts(BT, BC, float(z["clip"]))
    args = [torch.as_tensor(z[n]).cuda() for n in NAMES]
    h0 = torch.as_tensor(z["h0"]).cuda()
    o, h = gdn2_pallas_forward(*args, float(z["scale"]), h0)
    assert rel(o, z["o"]) < 1e-4 and rel(h, z["h_final"]) < 1e-4
    assert o.shape == (B, T, H, D) and h.shape == (B, H, D, D)
    # dk and dg are cancellation noise scaled by e^63 here (sign depends on
    # summation order): the remaining gradients are compared
    grads = dict(zip(GRADS, gdn2_backward(*args, float(z["scale"]), h0,
                                          torch.as_tensor(z["dout"]).cuda(),
                                          torch.as_tensor(z["dh_final"]).cuda())))
    for gname in ("dq", "dv", "dw", "db", "dh0"):
        assert rel(grads[gname], z[gname]) < 1e-4, (gname, rel(grads[gname], z[gname]))


def test_reference_shape_tests_on_gpu():
    """The reference's TPU shape tests (tests/test_pallas.py:14-41), on B200."""
    shape = (2, 512, 4, 128)
    ones = [torch.ones(shape, device="cuda") for _ in range(6)]
    out, h_final = gdn2_pallas_forward_trainable(*ones, 0.1)
    assert out.shape == shape and h_final.shape == (2, 4, 128, 128)
    out, _ = gdn2_pallas_forward(*ones, 0.1)
    assert out.shape == shape


def test_autograd_matches_direct_backward_and_recompute():
    _set_consts(128, 64, 1e3)
    inp = make_inputs(2, 512, 3, 128, seed=4, h0_std=0.1)
    leaves = [t.clone().requires_grad_(True) for t in _dev(inp, torch.float32)]
    h0 = torch.as_tensor(inp["h0"]).cuda().requires_grad_(True)
    do = torch.as_tensor(inp["dout"]).cuda()
    dhf = torch.as_tensor(inp["dh_final"]).cuda()
    o, h = gdn2_pallas_forward_trainable(*leaves, inp["scale"], h0)
    ((o * do).sum() + (h * dhf).sum()).backward()
    auto = [t.grad for t in leaves] + [h0.grad]
    direct = gdn2_backward(*[t.detach() for t in leaves], inp["scale"], h0.detach(), do, dhf)
    for name, a, b in zip(GRADS, auto, direct):
        assert torch.equal(a, b), name
    o2, h2 = gdn2_pallas_forward_trainable(*[t.detach() for t in leaves], inp["scale"],
                                           h0.detach(), recompute=True)
    assert torch.equal(o.detach(), o2) and torch.equal(h.detach(), h2)


def test_residuals_match_oracle_intermediates():
    _set_consts(64, 16, 1e4)
    inp = make_inputs(1, 256, 2, 64, seed=8, h0_std=0.1, grads=False)
    args = _dev(inp, torch.float32)
    o, h, res = gdn2_pallas_forward_with_residuals(*args, inp["scale"],
                                                   torch.as_tensor(inp["h0"]).cuda())
    _, _, r = O.forward(*[inp[n] for n in NAMES], inp["scale"], inp["h0"], 64, 16, 1e4,
                        residuals=True)
    for ours, theirs in [("Aqk", "Aqk"), ("A", "A"), ("w_pseudo", "W"), ("u", "U"), ("kg", "kg"),
                         ("qg", "qg"), ("gc_last", "gc_last"), ("h_pre_all", "h_pre"),
                         ("v_new_all", "v_new")]:
        assert rel(res[ours], r[theirs]) < 1e-5, ours


def test_host_buffers_round_trip():
    _set_consts(64, 16, 1e4)
    inp = make_inputs(1, 256, 2, 128, seed=9, grads=False)
    host = [torch.as_tensor(inp[n]).pin_memory() for n in NAMES]
    o, h = gdn2_pallas_forward(*host, inp["scale"])
    assert o.device.type == "cpu"
    o2, h2 = gdn2_pallas_forward(*[t.cuda() for t in host], inp["scale"])
    assert torch.equal(o, o2.cpu()) and torch.equal(h, h2.cpu())


def test_streaming_state_carry():
    """Processing T in two segments with h_final -> h0 equals one pass."""
    _set_consts(128, 64, 1e3)
    inp = make_inputs(2, 2048, 3, 128, seed=12, h0_std=0.1, grads=False)
    args = _dev(inp, torch.float32)
    h0 = torch.as_tensor(inp["h0"]).cuda()
    o, h = gdn2_pallas_forward(*args, inp["scale"], h0)
    o1, h1 = gdn2_pallas_forward(*[a[:, :1024] for a in args], inp["scale"], h0)
    o2, h2 = gdn2_pallas_forward(*[a[:, 1024:].contiguous() for a in args], inp["scale"], h1)
    assert rel(torch.cat([o1, o2], 1), o) < 1e-6 and rel(h2, h) < 1e-6


# ----------------------------------------------------------- benchmark sizes
def _full_check(B, T, H, D, BT, BC, clip, dtype, h0s=None, seed=0):
    _set_consts(BT, BC, clip)
    inp = make_inputs(B, T, H, D, seed=seed, h0_std=h0s)
    args = _dev(inp, dtype)
    h0 = torch.as_tensor(inp["h0"]).cuda() if "h0" in inp else None
    do = torch.as_tensor(inp["dout"]).cuda()
    dhf = torch.as_tensor(inp["dh_final"]).cuda()
    o, h = gdn2_pallas_forward_trainable(*args, inp["scale"], h0)
    grads = gdn2_backward(*args, inp["scale"], h0, do, dhf)
    ref_inp = {n: torch.as_tensor(inp[n]).to(dtype).double() for n in NAMES}
    ref_inp.update(scale=inp["scale"], h0=inp.get("h0"), dout=inp["dout"], dh_final=inp["dh_final"])
    o_r, h_r, g_r = torch_ref.forward_backward(ref_inp, BT, "cuda")
    tol = TOL[dtype]
    errs = {"o": rel(o, o_r), "h_final": rel(h, h_r)}
    errs.update({n: rel(a, b) for n, a, b in zip(GRADS, grads, g_r)})
    bad = {k: v for k, v in errs.items() if not v < tol}
    assert not bad, errs


def test_config1_full_size():
    """B=8 T=8192 H=6 D=128 fp32, BT=128 BC=64 CLIP=1e3 (the headline config)."""
    _full_check(8, 8192, 6, 128, 128, 64, 1e3, torch.float32)


def test_config2_full_size_bf16():
    """B=16 T=4096 H=16 D=128 bf16 inputs, BT=64 BC=16."""
    _full_check(16, 4096, 16, 128, 64, 16, 1e4, torch.bfloat16)


def test_config3_long_context():
    """B=1 T=131072 H=8 D=128 fp32, BT=128 BC=64 (single GPU)."""
    _full_check(1, 131072, 8, 128, 128, 64, 1e4, torch.float32)


def test_config4_forward_with_state():
    """B=64 T=2048 H=32 D=128 fp32 forward with h0 ~ N(0, 0.1), BT=64 BC=16.
    Inputs are drawn on the device; two batch slices are checked against the
    float64 reference (every (b, h) is independent), plus linearity in
    (v, h0)."""
    _set_consts(64, 16, 1e4)
    gen = torch.Generator(device="cuda").manual_seed(0)
    B, T, H, D = 64, 2048, 32, 128
    shp = (B, T, H, D)
    n = lambda s: torch.randn(s, device="cuda", generator=gen)
    q = torch.nn.functional.normalize(n(shp), dim=-1)
    k = torch.nn.functional.normalize(n(shp), dim=-1)
    v = n(shp)
    w = torch.sigmoid(n(shp))
    b = torch.sigmoid(n(shp))
    g = -torch.nn.functional.softplus(n(shp))
    h0 = 0.1 * n((B, H, D, D))
    scale = D ** -0.5
    o, h = gdn2_pallas_forward(q, k, v, w, b, g, scale, h0)
    for sl in (slice(0, 1), slice(B - 2, B)):
        o_r, h_r = torch_ref.forward(*[t[sl].double() for t in (q, k, v, w, b, g)], scale,
                                     h0[sl].double(), 64)
        assert rel(o[sl], o_r) < 1e-4 and rel(h[sl], h_r) < 1e-4
    o2, h2 = gdn2_pallas_forward(q, k, 2 * v, w, b, g, scale, 2 * h0)
    assert rel(o2, 2 * o) < 1e-5 and rel(h2, 2 * h) < 1e-5


@pytest.mark.parametrize("dtype,backward", [(torch.float32, True), (torch.bfloat16, True),
                                            (torch.float32, False)])
@pytest.mark.parametrize("shard,heads", [(1, 1), (1, 2), (5, 1), (1, None), (1, 4)])
def test_streamed_host_batches_equal_device_call(dtype, backward, shard, heads):
    """gdn2_fwd_bwd on host tensors ((batch rows x head group) shards moved
    by pitched copies through a ring of device buffers) gives the same bits
    as the device-resident call."""
    from gdn2_package import gdn2_fwd_bwd
    _set_consts(128, 64, 1e3)
    inp = make_inputs(5, 256, 4, 128, seed=17, h0_std=0.1)
    host = [torch.as_tensor(inp[n]).to(dtype).pin_memory() for n in NAMES]
    h0 = torch.as_tensor(inp["h0"])
    do = torch.as_tensor(inp["dout"]) if backward else None
    dhf = torch.as_tensor(inp["dh_final"]) if backward else None
    o, h, g = gdn2_fwd_bwd(*host, inp["scale"], do, dhf, h0, shard=shard, depth=2, heads=heads)
    assert o.device.type == "cpu"
    o2, h2, g2 = gdn2_fwd_bwd(*[t.cuda() for t in host], inp["scale"],
                              None if do is None else do.cuda(),
                              None if dhf is None else dhf.cuda(), h0.cuda())
    torch.cuda.synchronize()
    assert torch.equal(o, o2.cpu()) and torch.equal(h, h2.cpu())
    if backward:
        for a, b in zip(g, g2):
            assert a.dtype == b.dtype and torch.equal(a, b.cpu())
        ref = gdn2_backward(*[t.cuda() for t in host], inp["scale"], h0.cuda(), do.cuda(), dhf.cuda())
        for a, b in zip(g, ref):
            assert torch.equal(a, b.cpu())
    else:
        assert g is None


@pytest.mark.parametrize("BT,BC", [(128, 64), (64, 16)])
def test_stage_diagnostics_from_device_counters(BT, BC, monkeypatch, capsys):
    """GDN2_FWD_DIAG: every stage output the reference checks
    (gdn2_fwd.py:407-417) is reduced on the device.  Large values (v x 1e7,
    CLIP 1e9) are reported at kernel_C_u / kernel_D_h_final with the maxima of the
    stored tensors; an infinite q with CLIP = inf is reported non-finite at
    kernel_C_qg (qg = q e^gc keeps it)."""
    from gdn2_package import _lib
    monkeypatch.setattr(gdn2_fwd, "_GDN2_FWD_DIAG", True)
    _set_consts(BT, BC, 1e9)
    inp = make_inputs(1, 256, 2, 128, seed=23, h0_std=0.1, grads=False)
    inp["v"] = inp["v"] * np.float32(1e7)
    args = _dev(inp, torch.float32)
    o, h, res = gdn2_pallas_forward_with_residuals(*args, inp["scale"],
                                                   torch.as_tensor(inp["h0"]).cuda(),
                                                   debug_tag="t")
    out = capsys.readouterr().out
    assert "large value at t:kernel_C_u" in out and "large value at t:kernel_D_h_final" in out, out
    assert "t:kernel_A_Aqk" not in out and "non-finite" not in out, out
    from gdn2_package.gdn2_fwd import _Prepared, _run_forward
    p = _Prepared(*args, inp["scale"], torch.as_tensor(inp["h0"]).cuda())
    p.code |= _lib.NO_PAIR   # the kernels gdn2_pallas_forward_with_residuals ran
    o2, h2, ws = _run_forward(p, save_residuals=True, debug_tag="t")
    stats = _lib.diag_read(ws, p.stream)
    for tag, t in (("kernel_C_u", res["u"]), ("kernel_D_o", o2), ("kernel_D_h_final", h2),
                   ("kernel_A_Aqk", res["Aqk"]), ("kernel_C_kg", res["kg"])):
        assert stats[tag][0] == 0 and stats[tag][1] == float(t.abs().max()), (tag, stats[tag])
    capsys.readouterr()
    _set_consts(BT, BC, float("inf"))
    inp2 = make_inputs(1, 256, 2, 128, seed=24, grads=False)
    inp2["q"][0, 5, 1, 3] = np.inf
    gdn2_pallas_forward(*_dev(inp2, torch.float32), inp2["scale"], debug_tag="u")
    out = capsys.readouterr().out
    assert "non-finite at u:kernel_C_qg" in out, out


@pytest.mark.parametrize("BT,BC,dtype", [(128, 64, torch.float32), (64, 16, torch.float32),
                                         (128, 64, torch.bfloat16)])
def test_raw_gates_fused_into_the_loads(BT, BC, dtype, monkeypatch):
    """GATES = "raw": the kernels apply w = sigmoid(w'), b = sigmoid(b'),
    g = -softplus(g') as they load them, and return dw', db', dg'.  Checked
    against the float64 oracle on the activated inputs, with the chain rule
    applied to its gradients."""
    _set_consts(BT, BC, 1e3)
    inp = make_inputs(2, 256, 2, 128, seed=41, h0_std=0.1)
    rng = np.random.default_rng(5)
    raw = {n: rng.standard_normal(inp[n].shape).astype(np.float32) for n in ("w", "b", "g")}
    xs = dict(inp, **raw)
    args = [torch.as_tensor(xs[n]).cuda().to(dtype) for n in NAMES]
    h0 = torch.as_tensor(inp["h0"]).cuda()
    monkeypatch.setattr(gdn2_fwd, "GATES", "raw")
    o, h = gdn2_pallas_forward(*args, inp["scale"], h0)
    grads = gdn2_backward(*args, inp["scale"], h0, torch.as_tensor(inp["dout"]).cuda(),
                          torch.as_tensor(inp["dh_final"]).cuda())
    r = {n: torch.as_tensor(xs[n]).to(dtype).double().numpy() for n in NAMES}
    sig = lambda x: 1.0 / (1.0 + np.exp(-x))
    act = dict(r, w=sig(r["w"]), b=sig(r["b"]), g=-np.logaddexp(0.0, r["g"]))
    ref_in = [act[n] for n in NAMES]
    o_r, h_r = O.forward(*ref_in, inp["scale"], inp["h0"], BT, BC, 1e3)
    tol = TOL[dtype]
    assert rel(o, o_r) < tol and rel(h, h_r) < tol, (rel(o, o_r), rel(h, h_r))
    g_r = list(O.backward(*ref_in, inp["scale"], inp["h0"], inp["dout"], inp["dh_final"], BT, BC,
                          1e3))
    g_r[3] = g_r[3] * act["w"] * (1 - act["w"])          # dw'
    g_r[4] = g_r[4] * act["b"] * (1 - act["b"])          # db'
    g_r[5] = g_r[5] * -sig(r["g"])                        # dg'
    for name, a, b in zip(GRADS, grads, g_r):
        assert rel(a, b) < tol, (name, rel(a, b))
