"""gdn2_fwd_noalloc: the forward for callers that cannot allocate device
memory (for example a handler inside a framework that owns all device
allocations and passed no scratch buffer).  It must give the same results as
gdn2_fwd with a caller workspace, call after call, since every call reuses
the same built-in scratch array.  Collected last on purpose."""
import ctypes

import pytest
import torch

from conftest import cuda_ok
from gdn2_package import _lib
from gdn2_package.synthetic import make_inputs

NAMES = ("q", "k", "v", "w", "b", "g")


def _rel(a, b):
    return float((a.double() - b.double()).norm() / max(float(b.double().norm()), 1e-300))


def test_noalloc_rejects_oversized_problem_without_gpu_work():
    lib = _lib.load()
    dummy = ctypes.c_void_p(16)
    rc = lib.gdn2_fwd_noalloc(0, *[dummy] * 6, None, dummy, dummy,
                              64, 8192, 32, 128, 128, 64, 0.088, 1e4, None)
    assert rc == _lib.ERR_WORKSPACE
    assert "built-in limit" in lib.gdn2_last_error().decode()


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_ok(), reason="needs a CUDA device")
@pytest.mark.parametrize("B,T,H,D,BT,BC", [(1, 1024, 4, 128, 128, 64), (2, 512, 3, 64, 64, 16)])
def test_noalloc_matches_workspace_forward_twice(B, T, H, D, BT, BC):
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((21, 22)):   # two calls in a row, different inputs
        inp = make_inputs(B, T, H, D, seed=seed, h0_std=0.1, grads=False)
        x = [torch.as_tensor(inp[n]).cuda() for n in NAMES]
        h0 = torch.as_tensor(inp["h0"]).cuda()
        o_ref = torch.empty(B, T, H, D, device="cuda")
        h_ref = torch.empty(B, H, D, D, device="cuda")
        nbytes = lib.gdn2_workspace_bytes(B, T, H, D, BT, 0)
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        rc = lib.gdn2_fwd(0, *[t.data_ptr() for t in x], h0.data_ptr(), o_ref.data_ptr(),
                          h_ref.data_ptr(), ws.data_ptr(), nbytes, 0, B, T, H, D, BT, BC,
                          inp["scale"], 1e4, stream)
        assert rc == 0, lib.gdn2_last_error()
        o = torch.full((B, T, H, D), float("nan"), device="cuda")
        h = torch.full((B, H, D, D), float("nan"), device="cuda")
        rc = lib.gdn2_fwd_noalloc(0, *[t.data_ptr() for t in x], h0.data_ptr(), o.data_ptr(),
                                  h.data_ptr(), B, T, H, D, BT, BC, inp["scale"], 1e4, stream)
        assert rc == 0, lib.gdn2_last_error()
        torch.cuda.synchronize()
        assert _rel(o, o_ref) < 1e-4 and _rel(h, h_ref) < 1e-4, call
        # the call cleared the scratch's status header and no wait ran out
        assert lib.gdn2_noalloc_status(stream) == 0
