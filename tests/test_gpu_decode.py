"""Decode step (token-by-token with a carried state) against the float64
token recurrence of the oracle and against the chunked forward."""
import numpy as np
import pytest
import torch

from conftest import cuda_ok

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")]

import gdn2_oracle as O  # noqa: E402
from gdn2_package import gdn2_decode, gdn2_fwd, gdn2_pallas_forward  # noqa: E402
from gdn2_package.synthetic import make_inputs  # noqa: E402

NAMES = ("q", "k", "v", "w", "b", "g")


def rel(a, b):
    a = a.double().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_matches_token_recurrence(D, dtype):
    inp = make_inputs(2, 16, 3, D, seed=31, h0_std=0.1, grads=False)
    args = [torch.as_tensor(inp[n]).cuda().to(dtype) for n in NAMES]
    o, h = gdn2_decode(*args, inp["scale"], torch.as_tensor(inp["h0"]).cuda())
    ref = [torch.as_tensor(inp[n]).to(dtype).double().numpy() for n in NAMES]
    o_r, h_r = O.token_recurrence(*ref, inp["scale"], inp["h0"])
    tol = 1e-5 if dtype == torch.float32 else 1e-5   # the reference runs on the rounded inputs
    assert rel(o, o_r) < tol and rel(h, h_r) < tol, (rel(o, o_r), rel(h, h_r))


def test_decode_steps_chain_and_match_chunked_forward():
    """T single-token calls carrying h equal one T-token call, and both agree
    with the chunked forward on the same segment."""
    gdn2_fwd.BT, gdn2_fwd.BC = 64, 16
    inp = make_inputs(1, 64, 2, 128, seed=32, h0_std=0.1, grads=False)
    args = [torch.as_tensor(inp[n]).cuda() for n in NAMES]
    h0 = torch.as_tensor(inp["h0"]).cuda()
    o_all, h_all = gdn2_decode(*args, inp["scale"], h0)
    h, outs = h0, []
    for t in range(64):
        o_t, h = gdn2_decode(*[a[:, t:t + 1] for a in args], inp["scale"], h)
        outs.append(o_t)
    assert torch.equal(torch.cat(outs, 1), o_all) and torch.equal(h, h_all)
    o_c, h_c = gdn2_pallas_forward(*args, inp["scale"], h0)
    assert rel(o_all, o_c.double().cpu().numpy()) < 1e-5
    assert rel(h_all, h_c.double().cpu().numpy()) < 1e-5


def test_decode_rejects_bad_shapes():
    x = torch.zeros((1, 4, 2, 96), device="cuda")
    with pytest.raises(ValueError):
        gdn2_decode(x, x, x, x, x, x, 0.1)


@pytest.mark.parametrize("clip,gscale", [(0.3, 1.0), (1e4, 30.0)])
def test_decode_is_the_one_token_chunked_form(clip, gscale, monkeypatch):
    """Every sanitiser of the chunked form acts per token (W, U, kg, qg,
    gc_last, Aqk, o, h): equal to the oracle's chunked forward with BT = BC
    = 1, also with CLIP acting and with fast-decaying gates (g x 30, which
    exercise the exponential over its range)."""
    monkeypatch.setattr(gdn2_fwd, "CLIP", clip)
    inp = make_inputs(2, 24, 2, 128, seed=33, h0_std=0.1, grads=False)
    inp["g"] = inp["g"] * np.float32(gscale)
    args = [torch.as_tensor(inp[n]).cuda() for n in NAMES]
    o, h = gdn2_decode(*args, inp["scale"], torch.as_tensor(inp["h0"]).cuda())
    o_r, h_r = O.forward(*[inp[n].astype(np.float64) for n in NAMES], inp["scale"], inp["h0"],
                         1, 1, clip)
    assert rel(o, o_r) < 1e-5 and rel(h, h_r) < 1e-5, (rel(o, o_r), rel(h, h_r))


def test_decode_with_raw_gates(monkeypatch):
    """GATES = "raw": sigmoid / -softplus applied in the kernel equal the
    activations applied by the caller."""
    inp = make_inputs(1, 8, 2, 64, seed=34, h0_std=0.1, grads=False)
    raw = {n: torch.randn(inp[n].shape, generator=torch.Generator().manual_seed(i))
           for i, n in enumerate(("w", "b", "g"))}
    act = dict(w=torch.sigmoid(raw["w"]), b=torch.sigmoid(raw["b"]),
               g=-torch.nn.functional.softplus(raw["g"]))
    base = [torch.as_tensor(inp[n]) for n in ("q", "k", "v")]
    h0 = torch.as_tensor(inp["h0"]).cuda()
    o_a, h_a = gdn2_decode(*[t.cuda() for t in base + [act["w"], act["b"], act["g"]]],
                           inp["scale"], h0)
    monkeypatch.setattr(gdn2_fwd, "GATES", "raw")
    o_r, h_r = gdn2_decode(*[t.cuda() for t in base + [raw["w"], raw["b"], raw["g"]]],
                           inp["scale"], h0)
    assert rel(o_r, o_a.double().cpu().numpy()) < 1e-5 and rel(h_r, h_a.double().cpu().numpy()) < 1e-5
