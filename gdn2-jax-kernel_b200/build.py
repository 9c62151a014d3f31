"""Build libgdn2.so (sm_100a) in-tree with nvcc.

    python gdn2-jax-kernel_b200/build.py [--force]

Output: gdn2-jax-kernel_b200/gdn2_package/libgdn2.so.  nvcc cross-compiles
without a GPU, so this runs on any machine with the CUDA toolkit.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "gdn2_package", "libgdn2.so")
SOURCES = ["gdn2_fwd.cu", "gdn2_bwd.cu", "gdn2_capi.cu", "gdn2_selftest.cu", "gdn2_noalloc.cu", "gdn2_tc_kernels.cu", "gdn2_tc_bwd.cu", "gdn2_tc_fwd.cu", "gdn2_decode.cu", "gdn2_stages.cu"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo",
              "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def _nvcc():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _stale():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(ROOT, "include", "gdn2.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False):
    if not force and not _stale():
        return OUT
    objs = []
    bdir = os.path.join(HERE, "_build")
    os.makedirs(bdir, exist_ok=True)
    procs = []
    for src in SOURCES:
        obj = os.path.join(bdir, src.replace(".cu", ".o"))
        # GDN2_NVCC_EXTRA: extra flags, e.g. -DGDN2_PHASE_TIMING for the
        # per-phase cycle counts of the tensor-core kernels
        cmd = [_nvcc(), *NVCC_FLAGS, *os.environ.get("GDN2_NVCC_EXTRA", "").split(), "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    for cmd, p in procs:
        out = p.communicate()[0].decode()
        if verbose or p.returncode:
            sys.stderr.write(out)
        if p.returncode:
            raise RuntimeError("nvcc failed: " + " ".join(cmd))
    tmp = OUT + ".tmp"
    subprocess.check_call([_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
                           *objs, "-o", tmp, "-lcudart"])
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
