"""BT = 64 on the tensor-core kernels: two 64-row chunks per 128-row tile.

The paired tiles must compute the reference's BT = 64 function (block-
diagonal chunk scores and WY solve, gc, kg and gc_last per chunk, one state
step per chunk), so every check here is against the float64 oracle at
BT = 64, against the reference's own golden vectors, and against the
CUDA-core BT = 64 kernels on the same inputs.  Tolerances (rel-L2): 1e-4
for float32 inputs, 2e-2 for bfloat16.
"""
import os

import numpy as np
import pytest
import torch

import gdn2_oracle as O
from conftest import cuda_ok
from gdn2_package import _lib, gdn2_fwd, gdn2_pallas_forward
from gdn2_package.synthetic import make_inputs

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

NAMES = ("q", "k", "v", "w", "b", "g")
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def rel(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / max(float(b.norm()), 1e-300))


@pytest.fixture
def paired():
    lib = _lib.load()
    prev = lib.gdn2_pair64_enable(1)
    yield lib
    lib.gdn2_pair64_enable(prev)


def _set(BT, BC, clip):
    gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = BT, BC, clip


def _both_paths(lib, fn):
    """fn() with the paired tensor-core tiles, then with the CUDA-core kernels."""
    lib.gdn2_pair64_enable(1)
    a = fn()
    lib.gdn2_pair64_enable(0)
    b = fn()
    lib.gdn2_pair64_enable(1)
    return a, b


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,T,H,BC,h0s", [
    (1, 256, 2, 16, None),
    (2, 512, 3, 16, 0.1),
    (1, 384, 2, 32, 0.1),
    (1, 256, 2, 64, 0.1),
])
def test_forward_vs_oracle(paired, B, T, H, BC, h0s, dtype):
    _set(64, BC, 1e4)
    inp = make_inputs(B, T, H, 128, seed=5, h0_std=h0s)
    args = [torch.as_tensor(inp[n]).to("cuda", dtype) for n in NAMES]
    h0 = torch.as_tensor(inp["h0"]).cuda() if "h0" in inp else None
    (o, h), (o2, h2) = _both_paths(paired, lambda: gdn2_pallas_forward(*args, inp["scale"], h0))
    ref_in = [torch.as_tensor(inp[n]).to(dtype).double().numpy() for n in NAMES]
    o_r, h_r = O.forward(*ref_in, inp["scale"], inp.get("h0"), 64, BC, 1e4)
    tol = TOL[dtype]
    assert rel(o, o_r) < tol and rel(h, h_r) < tol, (rel(o, o_r), rel(h, h_r))
    # the two kernel families agree far inside the tolerance
    assert rel(o, o2) < 1e-5 and rel(h, h2) < 1e-5, (rel(o, o2), rel(h, h2))


@pytest.mark.parametrize("name", ["ref_bt64_bc32", "ref_ones_bt64_bc32"])
def test_forward_reference_golden(paired, name):
    """The reference source's own outputs; the all-ones case (g = +1) takes
    the exact elementwise scores with the +-20 clip and saturates CLIP."""
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    B, T, H, D, BT, BC = (int(x) for x in z["meta"])
    _set(BT, BC, float(z["clip"]))
    args = [torch.as_tensor(z[n]).cuda() for n in NAMES]
    h0 = torch.as_tensor(z["h0"]).cuda()
    o, h = gdn2_pallas_forward(*args, float(z["scale"]), h0)
    assert rel(o, z["o"]) < 1e-4 and rel(h, z["h_final"]) < 1e-4, (rel(o, z["o"]),
                                                                    rel(h, z["h_final"]))


@pytest.mark.parametrize("clip,h0s,gscale", [
    (0.3, 0.1, 1.0),     # U, W, kg, o clip
    (0.5, 0.1, 0.01),    # slow gates: the state itself clips between chunks
])
def test_forward_with_clip_active(paired, clip, h0s, gscale):
    """CLIP acting inside and between the two chunks of a tile: the state
    must be sanitised after each 64-row chunk, as the reference does."""
    _set(64, 16, clip)
    inp = make_inputs(2, 768, 2, 128, seed=31, h0_std=h0s)
    inp["g"] = inp["g"] * np.float32(gscale)
    args = [torch.as_tensor(inp[n]).cuda() for n in NAMES]
    h0 = torch.as_tensor(inp["h0"]).cuda()
    (o, h), (o2, h2) = _both_paths(paired, lambda: gdn2_pallas_forward(*args, inp["scale"], h0))
    o_r, h_r = O.forward(*[inp[n].astype(np.float64) for n in NAMES], inp["scale"], inp["h0"],
                         64, 16, clip)
    assert rel(o, o_r) < 1e-4 and rel(h, h_r) < 1e-4, (rel(o, o_r), rel(h, h_r))
    assert rel(o, o2) < 1e-5 and rel(h, h2) < 1e-5, (rel(o, o2), rel(h, h2))


GRADS = ("dq", "dk", "dv", "dw", "db", "dg", "dh0")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,T,H,BC,h0s", [
    (1, 256, 2, 16, None),
    (2, 512, 2, 32, 0.1),
    (1, 384, 2, 64, 0.1),
])
def test_backward_vs_oracle(paired, B, T, H, BC, h0s, dtype):
    from gdn2_package import gdn2_backward
    _set(64, BC, 1e4)
    inp = make_inputs(B, T, H, 128, seed=9, h0_std=h0s)
    args = [torch.as_tensor(inp[n]).to("cuda", dtype) for n in NAMES]
    h0 = torch.as_tensor(inp["h0"]).cuda() if "h0" in inp else None
    do = torch.as_tensor(inp["dout"]).cuda()
    dhf = torch.as_tensor(inp["dh_final"]).cuda()
    g1, g2 = _both_paths(paired, lambda: gdn2_backward(*args, inp["scale"], h0, do, dhf))
    ref_in = [torch.as_tensor(inp[n]).to(dtype).double().numpy() for n in NAMES]
    g_r = O.backward(*ref_in, inp["scale"], inp.get("h0"), inp["dout"], inp["dh_final"], 64, BC,
                     1e4)
    tol = TOL[dtype]
    for name, a, b, c in zip(GRADS, g1, g_r, g2):
        assert rel(a, b) < tol, (name, rel(a, b))
        assert rel(a, c) < (1e-5 if dtype == torch.float32 else 1e-2), (name, rel(a, c))


@pytest.mark.parametrize("name", ["ref_bt64_bc32", "ref_ones_bt64_bc32"])
def test_backward_reference_golden(paired, name):
    from gdn2_package import gdn2_backward
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    B, T, H, D, BT, BC = (int(x) for x in z["meta"])
    _set(BT, BC, float(z["clip"]))
    args = [torch.as_tensor(z[n]).cuda() for n in NAMES]
    h0 = torch.as_tensor(z["h0"]).cuda()
    grads = dict(zip(GRADS, gdn2_backward(*args, float(z["scale"]), h0,
                                          torch.as_tensor(z["dout"]).cuda(),
                                          torch.as_tensor(z["dh_final"]).cuda())))
    # all-ones: dk and dg are cancellation noise scaled by e^63 (their sign
    # depends on summation order), as in the reference's own comparison
    names = GRADS if name == "ref_bt64_bc32" else ("dq", "dv", "dw", "db", "dh0")
    for gname in names:
        assert rel(grads[gname], z[gname]) < 1e-4, (gname, rel(grads[gname], z[gname]))
    if name == "ref_ones_bt64_bc32":
        # g = +1: the call runs the float32 CUDA-core kernels (gdn2_fwd.PAIR64)
        paired.gdn2_pair64_enable(0)
        simt = gdn2_backward(*args, float(z["scale"]), h0, torch.as_tensor(z["dout"]).cuda(),
                             torch.as_tensor(z["dh_final"]).cuda())
        for gname, a in zip(GRADS, simt):
            assert torch.equal(a, grads[gname]), gname


def test_positive_gates_take_the_float32_kernels(paired):
    """A positive log-decay gate anywhere routes the whole call (forward and
    backward) to the CUDA-core kernels; g <= 0 pairs."""
    _set(64, 16, 1e4)
    inp = make_inputs(1, 256, 2, 128, seed=3)
    args = [torch.as_tensor(inp[n]).cuda() for n in NAMES]
    from gdn2_package import gdn2_fwd as F
    p = F._Prepared(*args, inp["scale"], None)
    assert not p.code & _lib.NO_PAIR
    args[5][0, 7, 1, 3] = 0.25
    p = F._Prepared(*args, inp["scale"], None)
    assert p.code & _lib.NO_PAIR
    (o, h), (o2, h2) = _both_paths(paired, lambda: gdn2_pallas_forward(*args, inp["scale"]))
    assert torch.equal(o, o2) and torch.equal(h, h2)


@pytest.mark.parametrize("BC", [16, 32])
@pytest.mark.parametrize("clip,dscale,h0s,gscale", [
    (20.0, 30.0, 0.1, 1.0),    # dv_new clips in the backward chain: exact recompute
    (0.3, 1.0, 0.1, 1.0),      # U, W, kg, o and the backward clip
    (0.5, 1.0, 0.1, 0.01),     # the forward state clips between the chunks of a tile
])
def test_backward_with_clip_active(paired, clip, dscale, h0s, gscale, BC, monkeypatch):
    """BC = 16 is guarded by the order-free bound of the B4 accumulators,
    BC = 32 by the block partials."""
    from gdn2_package import gdn2_backward
    monkeypatch.setattr(_lib, "CHECK_STATUS", "always")
    _set(64, BC, clip)
    inp = make_inputs(2, 768, 2, 128, seed=31, h0_std=h0s)
    inp["g"] = inp["g"] * np.float32(gscale)
    inp["dout"] = inp["dout"] * np.float32(dscale)
    inp["dh_final"] = inp["dh_final"] * np.float32(dscale)
    args = [torch.as_tensor(inp[n]).cuda() for n in NAMES]
    h0 = torch.as_tensor(inp["h0"]).cuda()
    grads = gdn2_backward(*args, inp["scale"], h0, torch.as_tensor(inp["dout"]).cuda(),
                          torch.as_tensor(inp["dh_final"]).cuda())
    assert _lib.LAST_STATUS & _lib.STATUS_EXACT_RECOMPUTE, _lib.LAST_STATUS
    g_r = O.backward(*[inp[n].astype(np.float64) for n in NAMES], inp["scale"], inp["h0"],
                     inp["dout"], inp["dh_final"], 64, BC, clip)
    for name, a, b in zip(GRADS, grads, g_r):
        assert rel(a, b) < 1e-4, (name, rel(a, b))


def test_trainable_keeps_residuals(paired):
    """The autograd path (forward keeping residuals, backward reading them)
    equals the backward that recomputes the forward, bit for bit."""
    from gdn2_package import gdn2_backward, gdn2_pallas_forward_trainable
    _set(64, 16, 1e4)
    inp = make_inputs(1, 512, 2, 128, seed=13, h0_std=0.1)
    args = [torch.as_tensor(inp[n]).cuda().requires_grad_() for n in NAMES]
    h0 = torch.as_tensor(inp["h0"]).cuda().requires_grad_()
    o, h = gdn2_pallas_forward_trainable(*args, inp["scale"], h0)
    do = torch.as_tensor(inp["dout"]).cuda()
    dhf = torch.as_tensor(inp["dh_final"]).cuda()
    torch.autograd.backward((o, h), (do, dhf))
    direct = gdn2_backward(*[a.detach() for a in args], inp["scale"], h0.detach(), do, dhf)
    for name, a, b in zip(GRADS, [*[a.grad for a in args], h0.grad], direct):
        assert torch.equal(a, b), name


@pytest.mark.parametrize("BT", [64, 128])
def test_b4_order_free_guard_bc16(paired, BT, monkeypatch):
    """BC = 16 below the score kernel's 32-column blocks: with nothing near
    CLIP the fast path runs (no B4 exact status) and matches the oracle; with
    CLIP small the guard sends the tiles to the pair-ordered path."""
    from gdn2_package import gdn2_backward
    monkeypatch.setattr(_lib, "CHECK_STATUS", "always")
    for clip in (1e4, 2.0):
        _set(BT, 16, clip)
        inp = make_inputs(1, 512, 2, 128, seed=41, h0_std=0.1)
        args = [torch.as_tensor(inp[n]).cuda() for n in NAMES]
        h0 = torch.as_tensor(inp["h0"]).cuda()
        grads = gdn2_backward(*args, inp["scale"], h0, torch.as_tensor(inp["dout"]).cuda(),
                              torch.as_tensor(inp["dh_final"]).cuda())
        exact_b4 = bool(_lib.LAST_STATUS & _lib.STATUS_B4_EXACT)
        assert exact_b4 == (clip < 1e4), (clip, _lib.LAST_STATUS)
        g_r = O.backward(*[inp[n].astype(np.float64) for n in NAMES], inp["scale"], inp["h0"],
                         inp["dout"], inp["dh_final"], BT, 16, clip)
        for name, a, b in zip(GRADS, grads, g_r):
            assert rel(a, b) < 1e-4, (clip, name, rel(a, b))
