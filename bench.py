"""Benchmark of the GDN-2 fwd+bwd hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (benchmark config 1): B=8 T=8192 H=6 D=128 fp32, BT=128 BC=64,
CLIP=1e3, synthetic inputs with the reference distributions (seed 0).  One
step = the trainable forward (keeping residuals) + the fused backward, i.e.
what ``gdn2_pallas_forward_trainable`` + ``.backward()`` run.  Under torchrun
every rank runs its own B=8 batch shard (batch x head sharding, no collective:
weak scaling); ``value`` is the tokens of all ranks / the slowest rank's time.

``--impl reference`` times the CPU restatement of the reference algorithm
(oracle/gdn2_oracle.py, float64 numpy) on the host cores: the reference
itself is JAX/Pallas-TPU code that cannot run on this machine.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "gdn2-jax-kernel_b200"))

CFG = dict(B=8, T=8192, H=6, D=128, BT=128, BC=64, CLIP=1e3)
METRIC = "fwd+bwd tokens/s at B8·T8192·H6·D128 fp32"
UNIT = "tokens/s"


def flops_per_chunk(C, D):
    """Algorithmic FLOPs of each kernel per (batch, head, chunk); a product
    with one triangular operand counts half of the dense 2mnk."""
    return {
        "fwd_intra": 4 * C * C * D + C ** 3 / 3,        # Aqk, Akk, (I+Akk)^-1, W, U
        "fwd_state": 6 * C * D * D + C * C * D,          # W h, qg h, kg^T vnew, Aqk vnew
        "bwd_state": 6 * C * D * D + C * C * D,          # kg dh, qg^T do, W^T dv, Aqk^T do
        "bwd_intra1": 8 * C * D * D + C * C * D,         # dv_new, dqg, dWp, dkg, dAqk
        "bwd_intra2": 6 * C * C * D + 4 * C ** 3 / 3,    # dA (2), dkb, dwv, dA A^T, A^T tmp
        "bwd_intra3": 4 * C * C * D,                     # four pair-sum products of B4
        "fwd_affine": 4 * C * D * D,                     # kg^T W, kg^T U
        "fwd_scan": 2 * D ** 3,                          # M h (serial)
        "fwd_out": 4 * C * D * D + C * C * D,            # W h, qg h, Aqk vnew
        "bwd_prep": 4 * C * D * D + C * C * D,           # Aqk^T do, qg^T do, W^T dvp
        "bwd_scan": 2 * D ** 3,                          # M^T dh (serial)
    }


def bytes_per_chunk(C, D):
    """Compulsory HBM bytes per chunk of each kernel (inputs it must read and
    outputs it must write, float32 workspace tiles included)."""
    t, s, cc = C * D * 4, D * D * 4, C * C * 4
    return {
        "fwd_intra": 6 * t + 2 * cc + 5 * t,
        "fwd_state": 4 * t + cc + 2 * t + s,
        "bwd_state": t + cc + 3 * t + t + s,
        "bwd_intra1": 2 * t + 3 * t + 2 * s + 3 * t + cc + 2 * t,   # + kg, dvp in, dv out, - dv in
        "bwd_intra2": 13 * t + 2 * cc,   # A, dAkk^T; dWp, dv, k, b, gc, w, v, pdk, pdgc in; pdk, pdb, pdgc, dw, dv out
        "bwd_intra3": 4 * t + 2 * cc + 5 * t + 4 * t,
        "fwd_affine": 3 * t + 2 * s,
        "fwd_scan": 3 * s,
        "fwd_out": 3 * t + s + cc + 3 * t,
        "bwd_prep": cc + 3 * t + t + s,
        "bwd_scan": 3 * s,
    }


# DRAM bytes (read + write) per chunk from one ncu capture of config 1 at B=1
# (384 chunks; traffic grows with the chunk count), profiles/tc_intra_kernels_config1_b1.md.
NCU_TRAFFIC_PER_CHUNK = {"fwd_intra": 743_297, "bwd_intra1": 970_652, "bwd_intra2": 1_199_843,
                         "bwd_intra3": 952_852}


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                  "sw_power_cap"), f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def _cpu_sample_worker(args):
    """One (batch, head) slice of length T_s through the oracle fwd+bwd;
    returns (tokens, seconds of compute)."""
    T_s, seed = args
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import gdn2_oracle as O
    from gdn2_package.synthetic import make_inputs
    inp = make_inputs(1, T_s, 1, CFG["D"], seed=seed)
    a = [inp[n] for n in ("q", "k", "v", "w", "b", "g")]
    t0 = time.perf_counter()
    O.forward(*a, inp["scale"], None, CFG["BT"], CFG["BC"], CFG["CLIP"])
    O.backward(*a, inp["scale"], None, inp["dout"], inp["dh_final"], CFG["BT"], CFG["BC"], CFG["CLIP"])
    return T_s, time.perf_counter() - t0


def _single_thread_env():
    for v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[v] = "1"


def run_reference(args, rank, world):
    if rank != 0:
        return
    import multiprocessing as mp
    _single_thread_env()
    procs = os.cpu_count() or 1
    T_s = 1024
    vals, wall = [], 0.0
    with mp.get_context("spawn").Pool(procs) as pool:
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            res = pool.map(_cpu_sample_worker, [(T_s, 100 + j) for j in range(procs)])
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                vals.append(sum(r[0] for r in res) / max(r[1] for r in res))
                wall += dt
    value = statistics.median(vals)
    sample = (f"each step: {procs} processes, each one (batch, head) slice of T={T_s} "
              "(float64 numpy oracle, fwd+bwd); tokens / slowest worker's compute time")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wall / max(args.steps, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (reference distributions, seeded)",
        "config": {"workload": "config1 fwd+bwd B8 T8192 H6 D128 BT128 BC64 CLIP1e3",
                   "sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": procs, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is JAX/Pallas-TPU code and JAX is not installed here; the timed "
                "arm is the CPU restatement of its algorithm",
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from gdn2_package import _lib, gdn2_fwd, gdn2_pipeline
    from gdn2_package.synthetic import make_inputs

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    B, T, H, D, BT = args.batch, CFG["T"], CFG["H"], CFG["D"], CFG["BT"]
    gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = BT, CFG["BC"], CFG["CLIP"]
    inp = make_inputs(B, T, H, D, seed=rank)
    names = ("q", "k", "v", "w", "b", "g")
    host = {n: torch.from_numpy(inp[n]).pin_memory() for n in names + ("dout", "dh_final")}
    devt = {n: t.to(dev) for n, t in host.items()}
    scale = inp["scale"]

    def step(d):
        (o, h), res = gdn2_pipeline._gdn2_core_fwd(*[d[n] for n in names], scale, None)
        grads = gdn2_pipeline._gdn2_core_bwd(scale, res, (d["dout"], d["dh_final"]))
        return o, h, grads

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(devt)
    barrier()

    # ---- device-resident timed region (inputs in HBM, 1.2 GB > L2)
    _lib.profile_read(reset=True)
    _lib.profile_enable(True)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        barrier()
        ev0.record()
        for _ in range(args.steps):
            step(devt)
        ev1.record()
        barrier()
    _lib.profile_enable(False)
    ms = ev0.elapsed_time(ev1)
    prof = _lib.profile_read(reset=True)

    # ---- end-to-end through the public API with host buffers
    out_host = None
    h2d = sum(t.numel() * t.element_size() for t in host.values())

    def e2e_step():
        nonlocal out_host
        d = {n: t.to(dev, non_blocking=True) for n, t in host.items()}
        o, h, grads = step(d)
        outs = [o, h, *grads]
        if out_host is None:
            out_host = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outs]
        for hb, t in zip(out_host, outs):
            hb.copy_(t, non_blocking=True)
        return outs

    e2e_ms, d2h = float("nan"), 0
    if not args.skip_e2e:
        outs = e2e_step()
        torch.cuda.synchronize()
        d2h = sum(t.numel() * t.element_size() for t in outs)
        e2e_steps = max(1, min(args.steps, 5))
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(e2e_steps):
            e2e_step()
        e1.record()
        barrier()
        e2e_ms = e0.elapsed_time(e1) / e2e_steps

    t = torch.tensor([ms, e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(t[0]), float(t[1])
    if rank != 0:
        return

    tokens = B * T * world
    ms_step = ms / args.steps
    nchunks = B * H * (T // BT)
    fl, by = flops_per_chunk(BT, D), bytes_per_chunk(BT, D)
    per_kernel = {}
    for s, (tot, cnt) in prof.items():
        if cnt:
            avg = tot / cnt
            per_kernel[s] = {"avg_ms": avg, "launches": cnt,
                             "tflops": fl[s] * nchunks / (avg * 1e-3) / 1e12,
                             "gbs": by[s] * nchunks / (avg * 1e-3) / 1e9}
    top = max(per_kernel, key=lambda s: per_kernel[s]["avg_ms"])
    hbm, tflops, kind = _peaks()
    tk = per_kernel[top]
    # Every intra-chunk kernel has ~11 algorithmic FLOP per byte, far under
    # the tensor ridge point (bf16 peak / HBM peak ~ 250 FLOP/B): HBM bounds them.
    traffic = NCU_TRAFFIC_PER_CHUNK.get(top)
    roofline = {"kernel": top, "bound": "hbm", "achieved": tk["gbs"], "peak": hbm,
                "unit": "GB/s", "frac": tk["gbs"] / hbm,
                "traffic": traffic * nchunks if traffic else None,
                "algorithmic_bytes": by[top] * nchunks, "peak_kind": kind + " copy bandwidth",
                "tensor_achieved_tflops": tk["tflops"], "tensor_peak_tflops": tflops,
                "tensor_frac": tk["tflops"] / tflops}
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        _single_thread_env()
        tok, dt = _cpu_sample_worker((T, 1))
        cpu = {"value": tok / dt, "unit": UNIT, "cores": 1, "kind": "port",
               "sample": f"one (batch, head) slice of the workload, T={T}, through the float64 "
                         f"numpy oracle fwd+bwd on one core ({dt:.1f} s)"}
    line = {
        "metric": METRIC, "value": tokens / (ms_step * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (reference distributions, seeded); inputs in HBM (1.2 GB > L2)",
        "config": {"workload": f"config1 fwd+bwd B{B} T8192 H6 D128 BT128 BC64 CLIP1e3 per GPU",
                   "global_batch": B * world, "seq_len": T, "heads": H, "head_dim": D,
                   "parallelism": f"dp{world} (batch x head shards, no collective)",
                   "l2": "inputs larger than L2"},
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": sum(v["launches"] for v in per_kernel.values()),
        "roofline": roofline,
        "kernels": per_kernel,
        "cpu_baseline": cpu,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_sp(args, rank, world, local_rank):
    """Config 3 (B1 T131072 H8 D128 fp32, BT128 BC64) fwd+bwd, the sequence
    split over the ranks (strong scaling: the job is fixed)."""
    import torch
    import torch.distributed as dist
    from gdn2_package import gdn2_fwd
    from gdn2_package import sequence_parallel as SP
    from gdn2_package.synthetic import make_inputs

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    B, T, H, D = 1, 131072, 8, 128
    gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = 128, 64, 1e4
    L = T // world
    inp = make_inputs(B, L, H, D, seed=1000 + rank)
    names = ("q", "k", "v", "w", "b", "g")
    x = [torch.from_numpy(inp[n]).to(dev) for n in names]
    do = torch.from_numpy(inp["dout"]).to(dev)
    dhf = torch.from_numpy(inp["dh_final"]).to(dev)
    gather = SP.dist_gather() if world > 1 else (lambda t: [t])

    def step():
        o, hf, st = SP.sp_forward(*x, inp["scale"], None, rank, gather)
        return SP.sp_backward(st, do, dhf, gather)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        ev0.record()
        for _ in range(args.steps):
            step()
        ev1.record()
        barrier()
    t = torch.tensor([ev0.elapsed_time(ev1)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank != 0:
        return
    ms = float(t[0]) / args.steps
    line = {
        "metric": "fwd+bwd tokens/s at B1·T131072·H8·D128 fp32 (sequence parallel)",
        "value": B * T / (ms * 1e-3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (reference distributions, seeded)",
        "config": {"workload": "config3 fwd+bwd B1 T131072 H8 D128 BT128 BC64, sequence split "
                               f"into {world} segments", "parallelism": f"sp{world}"},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=CFG["B"],
                    help="per-GPU batch (profiling of smaller cases only; the benchmark is B=8)")
    ap.add_argument("--skip-e2e", action="store_true", help="profiling: skip the host-buffer leg")
    ap.add_argument("--mode", default="dp", choices=["dp", "sp"],
                    help="dp: config 1 per GPU (default); sp: config 3 (B1 T131072 H8) split "
                         "over the GPUs by sequence")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.mode == "sp":
        if world > 1:
            import torch
            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
        try:
            run_sp(args, rank, world, local_rank)
        finally:
            if world > 1:
                import torch.distributed as dist
                dist.destroy_process_group()
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
