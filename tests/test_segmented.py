"""Chunk-parallel scan on one GPU (gdn2_package/segmented.py).

CPU: the segment plan and the batched float64 compositions against the
per-segment folds of sequence_parallel.  GPU: the segmented trainable
forward/backward against the serial path (o, h_final and all seven
gradients), and a saturating input that must fall back to the serial path
and so equal it exactly.
"""
import pytest
import torch

from conftest import cuda_ok
from gdn2_package import segmented as SG
from gdn2_package import sequence_parallel as SP

NAMES = ("q", "k", "v", "w", "b", "g")


def _rel(a, b):
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / max(float(b.norm()), 1e-300))


def test_plan_segments():
    # config 3 (B1 T131072 H8) on 148 SMs: 16 segments of 64 chunks, 128 CTAs
    assert SG.plan_segments(1, 131072, 8, 128, 148) == 16
    # config 1 (B8 H6): 48 scans already occupy a third of the SMs
    assert SG.plan_segments(8, 8192, 6, 128, 148) == 1
    # B2 H8: 16 scans, 8 segments each (128 CTAs)
    assert SG.plan_segments(2, 65536, 8, 128, 148) == 8
    # too short for two segments of MIN_SEGMENT_CHUNKS chunks
    assert SG.plan_segments(1, 2048, 2, 128, 148) == 1
    # T not divisible into whole-chunk segments
    assert SG.plan_segments(1, 128 * 33, 1, 128, 148) == 1
    # many sequences: no room on the SMs
    assert SG.plan_segments(16, 65536, 16, 128, 148) == 1


def test_batched_composition_matches_fold():
    g = torch.Generator().manual_seed(3)
    B, S, H, D = 2, 4, 3, 8
    P = 0.3 * torch.randn((B * S, H, D, D), generator=g, dtype=torch.float64)
    c = torch.randn((B * S, H, D, D), generator=g, dtype=torch.float64)
    h0 = torch.randn((B, H, D, D), generator=g, dtype=torch.float64)
    starts, final = SG._compose_forward(P, c, h0, S)
    for bb in range(B):
        ref_s, ref_f = SP.compose_forward([P[bb * S + s] for s in range(S)],
                                          [c[bb * S + s] for s in range(S)], h0[bb])
        for s in range(S):
            assert torch.allclose(starts[bb * S + s], ref_s[s])
        assert torch.allclose(final[bb], ref_f)
    e = torch.randn((B * S, H, D, D), generator=g, dtype=torch.float64)
    dhf = torch.randn((B, H, D, D), generator=g, dtype=torch.float64)
    g_in, g0 = SG._compose_backward(P, e, dhf, S)
    for bb in range(B):
        ref_in, ref_0 = SP.compose_backward([P[bb * S + s] for s in range(S)],
                                            [e[bb * S + s] for s in range(S)], dhf[bb])
        for s in range(S):
            assert torch.allclose(g_in[bb * S + s], ref_in[s])
        assert torch.allclose(g0[bb], ref_0)


def _run(fn, inp, dev="cuda"):
    x = [torch.as_tensor(inp[n]).to(dev).requires_grad_(True) for n in NAMES]
    h0 = torch.as_tensor(inp["h0"]).to(dev).requires_grad_(True)
    do = torch.as_tensor(inp["dout"]).to(dev)
    dhf = torch.as_tensor(inp["dh_final"]).to(dev)
    o, hf = fn(*x, inp["scale"], h0)
    ((o * do).sum() + (hf * dhf).sum()).backward()
    return [o.detach(), hf.detach()] + [t.grad for t in x] + [h0.grad]


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
@pytest.mark.parametrize("B,T,H,S", [(1, 8192, 2, 2), (1, 8192, 2, 4), (2, 4096, 1, 2)])
def test_segmented_matches_serial(B, T, H, S):
    from gdn2_package import gdn2_fwd, gdn2_pallas_forward_trainable
    from gdn2_package.synthetic import make_inputs
    gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = 128, 64, 1e4
    inp = make_inputs(B, T, H, 128, seed=40 + S, h0_std=0.1)
    ref = _run(gdn2_pallas_forward_trainable, inp)
    seg = _run(lambda *a: SG.gdn2_segmented_forward_trainable(*a, segments=S), inp)
    names = ("o", "h_final", "dq", "dk", "dv", "dw", "db", "dg", "dh0")
    for name, a, b in zip(names, seg, ref):
        assert _rel(a, b) < 1e-4, (name, _rel(a, b))


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_segmented_saturation_falls_back():
    """With CLIP acting on the state the segment maps are not affine: the
    forward must detect it and take the serial path, equal to it bit for bit."""
    from gdn2_package import gdn2_fwd, gdn2_pallas_forward_trainable
    from gdn2_package.synthetic import make_inputs
    gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = 128, 64, 0.5
    inp = make_inputs(1, 4096, 1, 128, seed=7, h0_std=0.1)
    inp["g"] = inp["g"] * 0.01   # slow decay: the state grows past CLIP = 0.5
    x = [torch.as_tensor(inp[n]).cuda() for n in NAMES]
    assert SG.segmented_forward(*x, inp["scale"], torch.as_tensor(inp["h0"]).cuda(), 2) is None
    ref = _run(gdn2_pallas_forward_trainable, inp)
    seg = _run(lambda *a: SG.gdn2_segmented_forward_trainable(*a, segments=2), inp)
    for a, b in zip(seg, ref):
        assert torch.equal(a, b)
