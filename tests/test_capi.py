"""The C ABI (include/gdn2.h) on a machine without a GPU: the library loads,
exports every declared entry point, sizes workspaces, and rejects bad
arguments before touching the device (the reference raises AssertionError
for these, gdn2_fwd.py:145-146)."""
import ctypes
import os
import re

import pytest

from gdn2_package import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "gdn2.h")).read()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(gdn2_\w+)\(", src, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = _declared()
    assert {"gdn2_fwd", "gdn2_bwd", "gdn2_workspace_bytes"} <= set(names)
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, n
    assert lib.gdn2_abi_version() == _lib.ABI_VERSION


def test_workspace_bytes():
    lib = _lib.load()
    B, T, H, D, C = 8, 8192, 6, 128, 128
    nc = T // C
    fwd = (2 * C * C + 5 * C * D + D + 4 * D * D + C * D + 4) * 4 * B * H * nc + 512
    bwd = fwd + (2 * C * C + 7 * C * D + 2 * D * D) * 4 * B * H * nc
    assert lib.gdn2_workspace_bytes(B, T, H, D, C, 0) == fwd
    assert lib.gdn2_workspace_bytes(B, T, H, D, C, 1) == bwd
    assert lib.gdn2_workspace_bytes(B, 100, H, D, C, 0) == 0


def _fwd(**kw):
    a = dict(dtype=0, B=1, T=128, H=1, D=64, BT=64, BC=16, scale=0.125, clip=1e4, ws=1 << 30)
    a.update(kw)
    lib = _lib.load()
    dummy = ctypes.c_void_p(16)
    rc = lib.gdn2_fwd(a["dtype"], *[dummy] * 6, None, dummy, dummy, dummy, a["ws"], 0,
                      a["B"], a["T"], a["H"], a["D"], a["BT"], a["BC"], a["scale"], a["clip"], None)
    return rc, lib.gdn2_last_error().decode()


@pytest.mark.parametrize("kw,frag", [
    (dict(D=96), "head dim"), (dict(BT=32), "chunk BT"), (dict(T=100), "divisible"),
    (dict(BC=48), "sub-block"), (dict(BC=8), "multiple of MB"), (dict(dtype=7), "dtype"),
    (dict(clip=0.0), "clip"),
    (dict(B=0), "empty"),
])
def test_invalid_arguments_rejected(kw, frag):
    rc, msg = _fwd(**kw)
    assert rc == _lib.ERR_INVALID and frag in msg


def test_small_workspace_rejected():
    rc, msg = _fwd(ws=1024)
    assert rc == _lib.ERR_WORKSPACE and "workspace too small" in msg


def test_python_api_shape_errors_match_reference_assertions():
    import torch
    from gdn2_package import gdn2_fwd, gdn2_pallas_forward
    x = torch.zeros(1, 100, 2, 64)
    with pytest.raises(AssertionError, match="divisible"):
        gdn2_pallas_forward(x, x, x, x, x, x, 0.1)
    gdn2_fwd.BT = 64
    y = torch.zeros(1, 128, 2, 96)
    with pytest.raises(ValueError, match="head dim"):
        gdn2_pallas_forward(y, y, y, y, y, y, 0.1)


def test_status_bits_match_header():
    src = open(os.path.join(ROOT, "include", "gdn2.h")).read()
    bits = dict(re.findall(r"#define GDN2_STATUS_(\w+) (\d+)", src))
    assert int(bits["WAIT_TIMEOUT"]) == _lib.STATUS_WAIT_TIMEOUT
    assert int(bits["FWD_STATE_CLIPPED"]) == _lib.STATUS_FWD_STATE_CLIPPED
    assert int(bits["BWD_STATE_CLIPPED"]) == _lib.STATUS_BWD_STATE_CLIPPED
    assert int(bits["EXACT_RECOMPUTE"]) == _lib.STATUS_EXACT_RECOMPUTE
    assert int(bits["B4_EXACT"]) == _lib.STATUS_B4_EXACT


def test_dtype_flags_match_header():
    src = open(os.path.join(ROOT, "include", "gdn2.h")).read()
    flags = dict(re.findall(r"#define GDN2_(GATES_RAW|NO_PAIR|NO_OUT) (0x[0-9a-f]+)", src))
    assert int(flags["GATES_RAW"], 16) == _lib.GATES_RAW
    assert int(flags["NO_PAIR"], 16) == _lib.NO_PAIR
    assert int(flags["NO_OUT"], 16) == _lib.NO_OUT


def test_no_out_needs_the_tensor_core_path_without_gpu_work():
    """GDN2_NO_OUT leaves o to a rescan that only the BT = D = 128 path has:
    elsewhere (and without saved residuals) the call is refused before any
    launch."""
    lib = _lib.load()
    fake = ctypes.c_void_p(256)
    args = [fake] * 6 + [None, None, fake, fake, 1 << 30]
    rc = lib.gdn2_fwd(_lib.F32 | _lib.NO_OUT, *args, 1, 1, 128, 2, 64, 64, 16, 0.1, 1e3, None)
    assert rc == _lib.ERR_INVALID
    assert "NO_OUT" in lib.gdn2_last_error().decode()
    rc = lib.gdn2_fwd(_lib.F32 | _lib.NO_OUT, *args, 0, 1, 128, 2, 128, 128, 64, 0.1, 1e3, None)
    assert rc == _lib.ERR_INVALID


def test_status_query_rejects_bad_workspace_without_gpu_work():
    lib = _lib.load()
    assert lib.gdn2_workspace_status(None, 1 << 20, None) == _lib.ERR_INVALID
    assert lib.gdn2_workspace_status(ctypes.c_void_p(256), 16, None) == _lib.ERR_INVALID
    assert lib.gdn2_selftest_wait_timeout(None, 1 << 20, 16, None) == _lib.ERR_INVALID


def test_copy_heads_rejects_bad_ranges_without_gpu_work():
    lib = _lib.load()
    h, d = ctypes.c_void_p(4096), ctypes.c_void_p(8192)
    assert lib.gdn2_copy_heads(None, d, 4, 6, 0, 3, 512, 1, None) == _lib.ERR_INVALID
    assert lib.gdn2_copy_heads(h, d, 4, 6, 4, 3, 512, 1, None) == _lib.ERR_INVALID   # 4+3 > 6
    assert lib.gdn2_copy_heads(h, d, 4, 6, 0, 0, 512, 0, None) == _lib.ERR_INVALID
    assert lib.gdn2_copy_heads(h, d, 4, 6, 0, 2, 0, 0, None) == _lib.ERR_INVALID
    assert lib.gdn2_copy_heads(h, d, 0, 6, 0, 2, 512, 0, None) == _lib.OK            # nothing to move


def test_stage_entry_points_reject_bad_arguments_without_gpu_work():
    lib = _lib.load()
    p = ctypes.c_void_p(4096)
    assert lib.gdn2_stage_scores(0, None, p, p, p, p, p, 1, 128, 1, 128, 64, 0.1, 1e4, None) \
        == _lib.ERR_INVALID
    assert lib.gdn2_stage_scores(0, p, p, p, p, p, p, 1, 128, 1, 128, 512, 0.1, 1e4, None) \
        == _lib.ERR_INVALID                                   # BT 64, 128 or 256
    assert lib.gdn2_stage_wy_solve(p, p, p, 4, 64, 8, 1e4, None) == _lib.ERR_INVALID   # BC % 16
    assert lib.gdn2_stage_wy_solve(p, p, None, 4, 256, 128, 1e4, None) == _lib.ERR_INVALID  # scratch
    assert lib.gdn2_stage_revcumsum(None, p, 4, 64, 128, 1e4, None) == _lib.ERR_INVALID
    assert lib.gdn2_stage_dav(p, p, p, p, p, 0, 64, 128, 1e4, None) == _lib.ERR_INVALID
    assert b"gdn2_stage" in lib.gdn2_last_error()


def test_stage_functions_have_the_reference_names():
    """gdn2_pipeline.py:14-31 imports these from gdn2_fwd / gdn2_bwd."""
    from gdn2_package import gdn2_bwd, gdn2_fwd
    for n in ("build_chunk_scores_pallas", "wy_solve_pallas", "recompute_wy_pallas",
              "gdn2_inter_chunk_combine", "gdn2_inter_chunk_combine_with_state"):
        assert callable(getattr(gdn2_fwd, n)), n
    for n in ("reverse_cumsum_bwd", "gdn2_dhu_backward", "dav_backward_pallas",
              "wy_dqkg_backward_pallas", "intra_backward_pallas"):
        assert callable(getattr(gdn2_bwd, n)), n
    gdn2_fwd.BT = 512
    try:
        with pytest.raises(gdn2_fwd.Gdn2ShapeError):
            gdn2_fwd._stage_bt()
    finally:
        gdn2_fwd.BT = 256


def test_streamed_shard_plan_covers_every_head_once():
    from gdn2_package.streaming import _shard_plan
    for B, H, Bs, Hs, edges in [(8, 6, 1, 3, True), (8, 6, 1, 3, False), (4, 4, 2, 2, True),
                                (1, 6, 1, 6, True), (2, 1, 1, 1, True)]:
        plan = _shard_plan(B, H, Bs, Hs, edges)
        cells = [(b, h) for b0, h0, hs in plan for b in range(b0, b0 + Bs) for h in range(h0, h0 + hs)]
        assert sorted(cells) == [(b, h) for b in range(B) for h in range(H)], (B, H, Bs, Hs, edges)
        if edges and Hs > 1 and B * H // (Bs * Hs) > 2:
            assert plan[0][2] == 1 and plan[-1][2] == 1 and plan[Hs][2] == Hs
    assert len(_shard_plan(8, 6, 1, 3, True)) == 16 - 2 + 6


def test_streamed_head_group_fills_the_gpu():
    from gdn2_package.streaming import _head_group
    assert _head_group(1, 8192, 6) == 3      # 64 chunks x 3 heads >= 148 CTAs
    assert _head_group(1, 32768, 6) == 1
    assert _head_group(2, 8192, 6) == 2
    assert _head_group(1, 256, 4) == 4       # never fills: the whole head range


def test_check_status_modes(monkeypatch):
    """The Python layer reads the status word only where its mode says, and a
    timed-out wait raises Gdn2Error (the read itself faked: no GPU here)."""
    seen = []
    monkeypatch.setattr(_lib, "workspace_status", lambda ws, s: seen.append(1) or 1)
    monkeypatch.setattr(_lib, "CHECK_STATUS", "sync")
    _lib.check_status(None, None, "x", synced=False)
    assert not seen
    with pytest.raises(_lib.Gdn2Error, match="timed out"):
        _lib.check_status(None, None, "x", synced=True)
    monkeypatch.setattr(_lib, "CHECK_STATUS", "never")
    _lib.check_status(None, None, "x", synced=True)
    assert len(seen) == 1
    monkeypatch.setattr(_lib, "CHECK_STATUS", "always")
    with pytest.raises(_lib.Gdn2Error):
        _lib.check_status(None, None, "x", synced=False)
