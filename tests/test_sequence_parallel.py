"""Sequence parallelism (gdn2_package/sequence_parallel.py).

CPU: the float64 composition of segment maps against a serial fold, and the
same through a 2-process gloo all-gather.  GPU: R ranks emulated on one
device (the exchange replaced by lists) against the full-sequence result, and
a real 2-GPU NCCL run when two devices are present.
"""
import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT, cuda_ok
from gdn2_package import sequence_parallel as SP

NAMES = ("q", "k", "v", "w", "b", "g")


def _rel(a, b):
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / max(float(b.norm()), 1e-300))


def test_compose_matches_serial_fold():
    g = torch.Generator().manual_seed(0)
    R, shape = 4, (2, 3, 8, 8)
    maps = [0.3 * torch.randn(shape, generator=g, dtype=torch.float64) for _ in range(R)]
    consts = [torch.randn(shape, generator=g, dtype=torch.float64) for _ in range(R)]
    h0 = torch.randn(shape, generator=g, dtype=torch.float64)
    starts, final = SP.compose_forward(maps, consts, h0)
    h = h0
    for r in range(R):
        assert torch.allclose(starts[r], h)
        h = maps[r] @ h + consts[r]
    assert torch.allclose(final, h)
    terms = [torch.randn(shape, generator=g, dtype=torch.float64) for _ in range(R)]
    gf = torch.randn(shape, generator=g, dtype=torch.float64)
    g_in, g0 = SP.compose_backward(maps, terms, gf)
    gg = gf
    for r in range(R - 1, -1, -1):
        assert torch.allclose(g_in[r], gg)
        gg = maps[r].transpose(-1, -2) @ gg + terms[r]
    assert torch.allclose(g0, gg)


_GLOO_WORKER = r'''
import os, sys, torch, torch.distributed as dist
sys.path.insert(0, os.path.join(sys.argv[1], "gdn2-jax-kernel_b200"))
from gdn2_package import sequence_parallel as SP
dist.init_process_group("gloo")
r, R = dist.get_rank(), dist.get_world_size()
gen = torch.Generator().manual_seed(100)
shape = (1, 2, 4, 4)
allP = [0.5 * torch.randn(shape, generator=gen) for _ in range(R)]
allc = [torch.randn(shape, generator=gen) for _ in range(R)]
gather = SP.dist_gather()
maps, consts = gather(allP[r]), gather(allc[r])
starts, final = SP.compose_forward(maps, consts, torch.zeros(shape))
ref_s, ref_f = SP.compose_forward(allP, allc, torch.zeros(shape))
assert all(torch.allclose(a, b) for a, b in zip(starts, ref_s)) and torch.allclose(final, ref_f)
dist.destroy_process_group()
open(os.path.join(sys.argv[2], f"ok{r}"), "w").close()   # one marker file per rank
'''


def test_exchange_over_gloo_two_ranks(tmp_path):
    script = tmp_path / "w.py"
    script.write_text(_GLOO_WORKER)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", "29533", str(script), ROOT,
           str(tmp_path)]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=240)
    assert out.returncode == 0, out.stderr[-2000:]
    assert (tmp_path / "ok0").exists() and (tmp_path / "ok1").exists()


def _inputs(B, T, H, seed):
    from gdn2_package.synthetic import make_inputs
    return make_inputs(B, T, H, 128, seed=seed, h0_std=0.1)


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
@pytest.mark.parametrize("R", [2, 4])
def test_sp_emulated_matches_full_sequence(R):
    from gdn2_package import gdn2_backward, gdn2_fwd, gdn2_pallas_forward
    gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = 128, 64, 1e4
    B, T, H = 1, 2048, 2
    inp = _inputs(B, T, H, 5)
    x = [torch.as_tensor(inp[n]).cuda() for n in NAMES]
    h0 = torch.as_tensor(inp["h0"]).cuda()
    do = torch.as_tensor(inp["dout"]).cuda()
    dhf = torch.as_tensor(inp["dh_final"]).cuda()
    o_ref, h_ref = gdn2_pallas_forward(*x, inp["scale"], h0)
    g_ref = gdn2_backward(*x, inp["scale"], h0, do, dhf)
    L = T // R
    seg = lambda t, r: t[:, r * L:(r + 1) * L].contiguous()
    states, Ps, cs = [], [], []
    for r in range(R):
        st, P, c = SP.sp_forward_local(*[seg(t, r) for t in x], inp["scale"], r)
        states.append(st); Ps.append(P); cs.append(c)
    outs = [SP.sp_forward_finish(st, Ps, cs, h0) for st in states]
    o = torch.cat([o_ for o_, _ in outs], 1)
    assert _rel(o, o_ref) < 1e-4 and _rel(outs[-1][1], h_ref) < 1e-4
    es = [SP.sp_backward_local(st, seg(do, r)) for r, st in enumerate(states)]
    grads = [SP.sp_backward_finish(st, es, dhf) for st in states]
    for i, name in enumerate(("dq", "dk", "dv", "dw", "db", "dg")):
        full = torch.cat([gr[i] for gr in grads], 1)
        assert _rel(full, g_ref[i]) < 1e-4, name
    assert _rel(grads[0][6], g_ref[6]) < 1e-4


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
def test_sp_reports_saturation():
    """A CLIP that acts on the state inside a segment makes the segment map
    non-affine: the ranks see it in the status bits and raise instead of
    returning a composition that differs from the serial scan."""
    from gdn2_package import gdn2_fwd
    gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = 128, 64, 0.5
    R, B, T, H = 2, 1, 512, 1
    inp = _inputs(B, T, H, 6)
    inp["g"] = inp["g"] * 0.01   # slow decay: the state grows past CLIP = 0.5
    x = [torch.as_tensor(inp[n]).cuda() for n in NAMES]
    L = T // R
    seg = lambda t, r: t[:, r * L:(r + 1) * L].contiguous()
    states, Ps, cs = [], [], []
    for r in range(R):
        st, P, c = SP.sp_forward_local(*[seg(t, r) for t in x], inp["scale"], r)
        states.append(st); Ps.append(P); cs.append(c)
    for st in states:
        SP.sp_forward_finish(st, Ps, cs, None)
    bits = [st.bits for st in states]
    assert any(b & SP._lib.STATUS_FWD_STATE_CLIPPED for b in bits), bits
    emulated = lambda t: [torch.tensor([b], dtype=torch.int32) for b in bits]
    with pytest.raises(SP.Gdn2SaturationError):
        SP._check_linear(bits[0], states[0].p, emulated, "sp_forward")


_NCCL_WORKER = r'''
import os, sys, torch, torch.distributed as dist
sys.path.insert(0, os.path.join(sys.argv[1], "gdn2-jax-kernel_b200"))
from gdn2_package import gdn2_fwd, gdn2_pallas_forward_trainable
from gdn2_package import sequence_parallel as SP
from gdn2_package.synthetic import make_inputs
r = int(os.environ["LOCAL_RANK"]); torch.cuda.set_device(r)
dist.init_process_group("nccl", device_id=torch.device("cuda", r))
R = dist.get_world_size()
gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = 128, 64, 1e4
inp = make_inputs(1, 1024 * R, 2, 128, seed=9, h0_std=0.1)
names = ("q", "k", "v", "w", "b", "g")
full = [torch.as_tensor(inp[n]).cuda().requires_grad_(True) for n in names]
h0 = torch.as_tensor(inp["h0"]).cuda()
do = torch.as_tensor(inp["dout"]).cuda(); dhf = torch.as_tensor(inp["dh_final"]).cuda()
o_ref, h_ref = gdn2_pallas_forward_trainable(*full, inp["scale"], h0)
((o_ref * do).sum() + (h_ref * dhf).sum()).backward()
L = 1024
loc = [t.detach()[:, r * L:(r + 1) * L].contiguous().requires_grad_(True) for t in full]
o, hf = SP.gdn2_sp_forward_trainable(*loc, inp["scale"], h0)
((o * do[:, r * L:(r + 1) * L]).sum() + (hf * dhf).sum()).backward()
rel = lambda a, b: float((a - b).norm() / b.norm())
errs = [rel(o, o_ref.detach()[:, r * L:(r + 1) * L]), rel(hf, h_ref.detach())]
errs += [rel(a.grad, b.grad[:, r * L:(r + 1) * L]) for a, b in zip(loc, full)]
assert max(errs) < 1e-4, errs
dist.destroy_process_group()
print("ok", r, max(errs))
'''


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sp_two_gpus_nccl(tmp_path):
    script = tmp_path / "w.py"
    script.write_text(_NCCL_WORKER)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", "29534", str(script), ROOT]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    assert "ok 0" in out.stdout and "ok 1" in out.stdout
