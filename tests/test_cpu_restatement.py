"""The fp32 C++/OpenMP restatement (oracle/gdn2_cpu.cpp, the benchmark's CPU
baseline) against the float64 oracle: forward and all seven gradients, with
and without CLIP acting, on both chunk lengths."""
import numpy as np
import pytest

import gdn2_cpu
import gdn2_oracle as O
from gdn2_package.synthetic import make_inputs

NAMES = ("q", "k", "v", "w", "b", "g")


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-300))


@pytest.mark.parametrize("BT,BC,D,clip,ds", [(64, 16, 64, 1e4, 1.0), (128, 64, 128, 1e3, 1.0),
                                             (128, 64, 128, 20.0, 30.0)])
def test_cpu_restatement_matches_oracle(BT, BC, D, clip, ds):
    inp = make_inputs(1, 256, 2, D, seed=5, h0_std=0.1)
    inp["dout"] = inp["dout"] * np.float32(ds)
    inp["dh_final"] = inp["dh_final"] * np.float32(ds)
    o, h, g = gdn2_cpu.fwd_bwd(inp, BT, BC, clip, threads=2)
    a = [inp[n].astype(np.float64) for n in NAMES]
    o_r, h_r = O.forward(*a, inp["scale"], inp["h0"], BT, BC, clip)
    g_r = O.backward(*a, inp["scale"], inp["h0"], inp["dout"], inp["dh_final"], BT, BC, clip)
    assert rel(o, o_r) < 1e-4 and rel(h, h_r) < 1e-4
    for x, y in zip(g, g_r):
        assert rel(x, y) < 1e-4
