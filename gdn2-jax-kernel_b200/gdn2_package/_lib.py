"""ctypes binding of libgdn2.so, the C ABI declared in include/gdn2.h.

The shared library is built in-tree (``gdn2-jax-kernel_b200/build.py``) and
loaded from this directory.  There is no fallback: if the library or a CUDA
device is missing, every call raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgdn2.so")

F32, BF16 = 0, 1
GATES_RAW = 0x100   # flag OR-ed into the dtype code (include/gdn2.h)
NO_PAIR = 0x200     # flag: BT = 64 on the CUDA-core kernels for this call
NO_OUT = 0x400      # flag: gdn2_fwd forms residuals and h_final, not o (a rescan follows)
OK, ERR_INVALID, ERR_WORKSPACE, ERR_CUDA = 0, -1, -2, -3
# bits of gdn2_workspace_status (include/gdn2.h)
STATUS_WAIT_TIMEOUT, STATUS_FWD_STATE_CLIPPED, STATUS_BWD_STATE_CLIPPED = 1, 2, 4
STATUS_EXACT_RECOMPUTE, STATUS_B4_EXACT = 8, 16
ABI_VERSION = 1

_lib = None

_vp, _i, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t

SIGNATURES = {
    "gdn2_abi_version": (_i, []),
    "gdn2_last_error": (ctypes.c_char_p, []),
    "gdn2_workspace_bytes": (_sz, [_i, _i, _i, _i, _i, _i]),
    "gdn2_fwd": (_i, [_i] + [_vp] * 6 + [_vp, _vp, _vp, _vp, _sz, _i] + [_i] * 6 + [_f, _f, _vp]),
    "gdn2_bwd": (_i, [_i] + [_vp] * 6 + [_vp, _vp, _vp] + [_vp] * 6 + [_vp, _vp, _sz, _i]
                 + [_i] * 6 + [_f, _f, _vp]),
    "gdn2_fwd_noalloc": (_i, [_i] + [_vp] * 6 + [_vp, _vp, _vp] + [_i] * 6 + [_f, _f, _vp]),
    "gdn2_decode": (_i, [_i] + [_vp] * 6 + [_vp, _vp, _vp] + [_i] * 4 + [_f, _f, _vp]),
    "gdn2_sp_segment": (_i, [_i, _vp, _sz, _vp, _vp, _vp] + [_i] * 6 + [_f, _f, _vp]),
    "gdn2_profile_enable": (_i, [_i]),
    "gdn2_selftest_gemm_tf32x3": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp]),
    "gdn2_profile_read": (_i, [_i, ctypes.POINTER(ctypes.c_double),
                               ctypes.POINTER(ctypes.c_long), _i]),
    "gdn2_workspace_status": (_i, [_vp, _sz, _vp]),
    "gdn2_noalloc_status": (_i, [_vp]),
    "gdn2_copy_heads": (_i, [_vp, _vp, ctypes.c_long, _i, _i, _i, _sz, _i, _vp]),
    "gdn2_selftest_wait_timeout": (_i, [_vp, _sz, _i, _vp]),
    "gdn2_diag_enable": (_i, [_i]),
    "gdn2_pair64_enable": (_i, [_i]),
    "gdn2_stage_scores": (_i, [_i] + [_vp] * 6 + [_i] * 5 + [_f, _f, _vp]),
    "gdn2_stage_wy_solve": (_i, [_vp, _vp, _vp, _i, _i, _i, _f, _vp]),
    "gdn2_stage_recompute_wy": (_i, [_i] + [_vp] * 12 + [_i] * 5 + [_f, _vp]),
    "gdn2_stage_combine": (_i, [_vp] * 11 + [_i] * 5 + [_f, _f, _vp]),
    "gdn2_stage_dhu": (_i, [_vp] * 10 + [_i] * 5 + [_f, _f, _vp]),
    "gdn2_stage_dav": (_i, [_vp] * 5 + [_i] * 3 + [_f, _vp]),
    "gdn2_stage_wy_dqkg": (_i, [_vp] * 20 + [_i] * 3 + [_f, _f, _vp]),
    "gdn2_stage_intra_bwd": (_i, [_i] + [_vp] * 11 + [_i] * 6 + [_f, _f, _vp]),
    "gdn2_stage_revcumsum": (_i, [_vp, _vp, _i, _i, _i, _f, _vp]),
    "gdn2_diag_read": (_i, [_vp, _sz, _vp, _i, ctypes.POINTER(ctypes.c_int),
                            ctypes.POINTER(ctypes.c_float)]),
}

# Stage tags of the forward diagnostics, in gdn2_diag_read's order
# (the reference's _stage_diag tags, gdn2_fwd.py:407-417, 360-363).
DIAG_STAGES = ("kernel_A_Aqk", "kernel_A_Akk", "kernel_B_wy_inverse_A", "kernel_C_w_pseudo",
               "kernel_C_u", "kernel_C_kg", "kernel_C_qg", "kernel_D_o", "kernel_D_h_final")


def diag_read(ws, stream):
    """{stage tag: (n_nonfinite, max_abs)} of the latest forward on ``ws``
    (diagnostics must have been enabled for that call).  Synchronizes."""
    n = len(DIAG_STAGES)
    nf = (ctypes.c_int * n)()
    mx = (ctypes.c_float * n)()
    rc = load().gdn2_diag_read(ws.data_ptr(), ws.numel(), stream, n, nf, mx)
    if rc < 0:
        check(rc, "gdn2_diag_read")
    return {t: (nf[i], mx[i]) for i, t in enumerate(DIAG_STAGES)}

STAGES = ("fwd_intra", "fwd_state", "bwd_state", "bwd_intra1", "bwd_intra2", "bwd_intra3",
          "fwd_affine", "fwd_scan", "fwd_out", "bwd_prep", "bwd_scan", "bwd_exact")


def profile_enable(on=True):
    load().gdn2_profile_enable(int(on))


def profile_read(reset=True):
    """{stage: (total_ms, launches)} of the launches timed since the last reset."""
    n = len(STAGES)
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_long * n)()
    load().gdn2_profile_read(n, ms, cnt, int(reset))
    return {s: (ms[i], cnt[i]) for i, s in enumerate(STAGES)}


class Gdn2Error(RuntimeError):
    """A CUDA-side failure reported by libgdn2."""


# When the device status word of a call is read back and checked:
#   "sync"   at the points where the package synchronizes anyway (calls made
#            with host tensors, whose results are copied back);
#   "always" after every call (one stream synchronization per call);
#   "never".
# The environment variable GDN2_CHECK_STATUS sets the initial mode.
CHECK_STATUS = os.environ.get("GDN2_CHECK_STATUS", "sync")
LAST_STATUS = None   # status bits of the latest call that was checked


def workspace_status(ws, stream):
    """The status bits of the latest call on workspace tensor ``ws``
    (STATUS_* above; 0 = nothing to report).  Synchronizes ``stream``."""
    rc = load().gdn2_workspace_status(ws.data_ptr(), ws.numel(), stream)
    if rc < 0:
        check(rc, "gdn2_workspace_status")
    return rc


def check_status(ws, stream, what, synced):
    """Raise Gdn2Error if the call that used ``ws`` recorded a timed-out wait.
    ``synced``: the caller synchronizes at this point anyway."""
    global LAST_STATUS
    if CHECK_STATUS == "always" or (CHECK_STATUS == "sync" and synced):
        LAST_STATUS = workspace_status(ws, stream)
        if LAST_STATUS & STATUS_WAIT_TIMEOUT:
            raise Gdn2Error(f"{what}: a bounded barrier wait inside a kernel timed out; "
                            "the results of this call are invalid")


def load():
    """Load (once) and return the ctypes handle of libgdn2.so."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libgdn2.so not found at {LIB_PATH}; build it with "
            "`python gdn2-jax-kernel_b200/build.py` (nvcc, sm_100a)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.gdn2_abi_version() != ABI_VERSION:
        raise ImportError("libgdn2.so ABI version mismatch; rebuild it")
    _lib = lib
    return lib


def check(rc, what):
    if rc == OK:
        return
    msg = load().gdn2_last_error().decode(errors="replace")
    if rc == ERR_INVALID:
        from .gdn2_fwd import Gdn2ShapeError
        raise Gdn2ShapeError(f"{what}: {msg}")
    raise Gdn2Error(f"{what} failed ({rc}): {msg}")
