"""Benchmark of the GDN-2 hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 1|2|3|4] [--scaling weak|strong] [--mode dp|sp]

Default workload: B=8 T=8192 H=6 D=128 fp32, BT=128
BC=64, CLIP=1e3, synthetic inputs with the reference distributions.  One step
= the trainable forward (keeping residuals) + the fused backward, i.e. what
``gdn2_pallas_forward_trainable`` + ``.backward()`` run.  ``--config`` picks
another BASELINE configuration (2: bf16 fwd+bwd B16 T4096 H16 BT64; 3: fp32
fwd+bwd B1 T131072 H8 on one GPU; 4: fp32 forward with h0, B64 T2048 H32
BT64).  Under torchrun every rank runs its own copy of the configuration
(``--scaling weak``, batch x head sharding with no collective) or one slice
of its (batch, head) units (``--scaling strong``); ``value`` is the tokens of
all ranks / the slowest rank's time.  ``--mode sp`` runs config 3 with the
sequence split over the ranks.

``--impl reference`` times the fp32 C++/OpenMP restatement of the reference
algorithm (oracle/gdn2_cpu.cpp, checked against the float64 oracle) on all
host cores: the reference itself is JAX/Pallas-TPU code that cannot run on
this machine.
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

CONFIGS = {   # BASELINE.json configs (config 0 is the oracle-only parity case)
    1: dict(B=8, T=8192, H=6, D=128, BT=128, BC=64, CLIP=1e3, dtype="f32", bwd=True, h0=None),
    2: dict(B=16, T=4096, H=16, D=128, BT=64, BC=16, CLIP=1e4, dtype="bf16", bwd=True, h0=None),
    3: dict(B=1, T=131072, H=8, D=128, BT=128, BC=64, CLIP=1e4, dtype="f32", bwd=True, h0=None),
    4: dict(B=64, T=2048, H=32, D=128, BT=64, BC=16, CLIP=1e4, dtype="f32", bwd=False, h0=0.1),
}
CFG = CONFIGS[1]
METRIC = "fwd+bwd tokens/s at B8·T8192·H6·D128 fp32"
UNIT = "tokens/s"


def metric_of(cfg):
    mode = "fwd+bwd" if cfg["bwd"] else "fwd"
    dt = "fp32" if cfg["dtype"] == "f32" else "bf16"
    return f"{mode} tokens/s at B{cfg['B']}·T{cfg['T']}·H{cfg['H']}·D{cfg['D']} {dt}"


def workload_of(cfg, n, note=""):
    mode = "fwd+bwd" if cfg["bwd"] else "fwd"
    h0 = f" h0~N(0,{cfg['h0']})" if cfg["h0"] else ""
    return (f"config{n} {mode} B{cfg['B']} T{cfg['T']} H{cfg['H']} D{cfg['D']} {cfg['dtype']} "
            f"BT{cfg['BT']} BC{cfg['BC']} CLIP{cfg['CLIP']:g}{h0}{note}")


def flops_per_chunk(C, D):
    """Algorithmic FLOPs of each kernel per (batch, head, chunk); a product
    with one triangular operand counts half of the dense 2mnk.  bwd_exact is
    the guard launch of the tensor-core backward: it does no work unless the
    guard flagged a (batch, head)."""
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
        "bwd_exact": 0,
    }


def bytes_per_chunk(C, D, s=4):
    """Compulsory HBM bytes per chunk of each kernel: the inputs it must read
    and the outputs it must write.  Workspace tiles are float32; the six
    input tensors and the six gradients have element size ``s``."""
    t, s2, cc = C * D * 4, D * D * 4, C * C * 4
    x = C * D * s   # one input or gradient tile
    return {
        "fwd_intra": 6 * x + 2 * cc + 5 * t,               # q k v w b g in; Aqk A W U kg qg gc out
        "fwd_state": 4 * t + cc + 2 * t + s2,              # W U kg qg Aqk in; o vnew out; h
        "bwd_state": t + cc + 3 * t + t + s2,
        "bwd_intra1": 2 * x + 3 * t + 2 * s2 + 3 * t + cc + 2 * t,   # q k, do vnew kg dvp, h dh; pdq pdk pdgc dAqk dWp dv
        "bwd_intra2": 4 * x + 2 * x + 7 * t + 2 * cc,      # k v w b in, dw dv out; A dAkk, dWp dv gc pdk pdgc in/out pdb
        "bwd_intra3": 4 * x + 2 * cc + 5 * t + 4 * x,      # q k b g; dAqk dAkk; gc pd*; dq dk db dg out
        "fwd_affine": 3 * t + 3 * s2,                      # kg W U in; M (both ways), Bc out
        "fwd_scan": 3 * s2,                                # M, Bc in; h out
        "fwd_out": 3 * t + s2 + cc + 3 * t,
        "bwd_prep": cc + 3 * t + t + s2,
        "bwd_scan": 3 * s2,                                # M^T, E in; dh out
        "bwd_exact": 0,
    }


def step_work(cfg):
    """Whole-step algorithmic FLOPs and compulsory HBM bytes (the per token
    and head figures of the benchmark spec): F_fwd = 5CD + 6D^2 + C^2/3,
    F_fwd+bwd = 15CD + 18D^2 + C^2; bytes (6s+4)D forward and (18s+8)D
    forward+backward, plus h0 / h_final."""
    C, D = cfg["BT"], cfg["D"]
    s = 4 if cfg["dtype"] == "f32" else 2
    th = cfg["B"] * cfg["T"] * cfg["H"]
    if cfg["bwd"]:
        f = 15 * C * D + 18 * D * D + C * C
        by = (18 * s + 8) * D
    else:
        f = 5 * C * D + 6 * D * D + C * C / 3
        by = (6 * s + 4) * D
    states = cfg["B"] * cfg["H"] * D * D * 4 * (2 if cfg["h0"] else 1)
    return f * th, by * th + states


# DRAM bytes (read + write) per chunk of config 1's kernels from one ncu
# capture at B=1 (384 chunks, inputs larger than L2); traffic grows with the
# chunk count, so a full launch moves this figure x 3072 chunks.
NCU_TRAFFIC_PER_CHUNK = {"fwd_intra": 738_587, "bwd_intra1": 960_509, "bwd_intra2": 1_199_761,
                         "bwd_intra3": 953_457}


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []
        self.n0 = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi prints its first sample as soon as it is up: wait for
            # it so that the samples cover the region that follows, and keep
            # only the later ones
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5 and self.proc.poll() is None:
                time.sleep(0.01)
            self.n0 = len(self.lines)
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
        for ln in self.lines[self.n0:] or self.lines:
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
    """(HBM GB/s, bf16 dense TFLOP/s burst, kind) from MEASURED_PEAKS.json."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def tensor_peak(cfg, bf16_tflops):
    """Logical TFLOP/s ceiling of the path a config runs on.  The chunk = head
    dim = 128 kernels compute every product as 3xTF32 (three kind::tf32 MMAs
    per logical product; dense TF32 runs at half the bf16 rate), so their
    ceiling is bf16 / 2 / 3.  The 64-row kernels run on the CUDA cores: 148
    SMs x 128 FMA/clk x 2 x 1.965 GHz.  BT = 64 with D = 128 runs the
    tensor-core kernels on tiles of two chunks (gdn2_fwd.PAIR64)."""
    if cfg["D"] == 128 and (cfg["BT"] == 128 or (cfg["BT"] == 64 and cfg["T"] % 128 == 0)):
        return bf16_tflops / 6.0, "3xTF32 logical = measured bf16 burst / 2 (TF32) / 3"
    return 148 * 128 * 2 * 1.965e9 / 1e12, "fp32 CUDA-core FMA (148 SMs x 128 x 2 x 1.965 GHz)"


def _cpu_inputs(cfg, slices, seed=100):
    from gdn2_package.synthetic import make_inputs
    return make_inputs(1, cfg["T"], slices, cfg["D"], seed=seed, h0_std=cfg["h0"],
                       grads=cfg["bwd"])


def _cpu_run(cfg, inp, threads):
    """One fwd(+bwd) of the fp32 C++/OpenMP restatement of the reference
    (oracle/gdn2_cpu.cpp) over the sample; returns seconds."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import gdn2_cpu
    t0 = time.perf_counter()
    gdn2_cpu.fwd_bwd(inp, cfg["BT"], cfg["BC"], cfg["CLIP"], threads=threads, backward=cfg["bwd"])
    return time.perf_counter() - t0


def _cpu_plan(cfg):
    """(slices, threads): one (batch, head) slice per host core, at most the
    configuration's B*H, each at the full T."""
    cores = os.cpu_count() or 1
    return min(cfg["B"] * cfg["H"], cores), cores


def _cpu_sample_text(cfg, slices, threads, dt=None):
    mode = "fwd+bwd" if cfg["bwd"] else "fwd"
    t = f" ({dt:.1f} s)" if dt is not None else ""
    return (f"{slices} of the {cfg['B'] * cfg['H']} (batch, head) slices of the workload at the "
            f"full T={cfg['T']}, {mode} (the forward recomputed in the backward, as the reference "
            f"does), fp32 C++/OpenMP restatement of the reference on {threads} threads{t}; "
            f"tokens = slices x T")


def run_reference(args, rank, world):
    """The reference's algorithm on the host cores: the fp32 C++/OpenMP
    restatement (oracle/gdn2_cpu.cpp) over one (batch, head) slice per core at
    the configuration's full length T; throughput = tokens of the sample /
    its wall time.  The reference itself is JAX/Pallas for TPU and cannot run
    here."""
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    slices, threads = _cpu_plan(cfg)
    inp = _cpu_inputs(cfg, slices)
    vals, wall = [], 0.0
    for i in range(args.warmup + args.steps):
        dt = _cpu_run(cfg, inp, threads)
        if i >= args.warmup:
            vals.append(slices * cfg["T"] / dt)
            wall += dt
    value = statistics.median(vals)
    sample = _cpu_sample_text(cfg, slices, threads)
    line = {
        "impl": "reference", "metric": METRIC if args.config == 1 else metric_of(cfg),
        "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wall / max(args.steps, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (reference distributions, seeded)",
        "config": {"workload": workload_of(cfg, args.config), "sample": sample,
                   "same_config": True},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is JAX/Pallas-TPU code and JAX is not installed here; the timed "
                "arm is an fp32 C++/OpenMP restatement of its algorithm, checked against the "
                "float64 oracle pinned to the reference's own outputs",
    }
    print(json.dumps(line), flush=True)


def _shard(cfg, world, rank, scaling):
    """Per-rank (B, H) of the job.  weak: every rank runs the whole
    configuration; strong: the configuration's (batch, head) units are split
    over the ranks (batch first, then heads)."""
    B, H = cfg["B"], cfg["H"]
    if scaling == "weak" or world == 1:
        return B, H
    if B % world == 0:
        return B // world, H
    if H % world == 0:
        return B, H // world
    raise SystemExit(f"strong scaling: B={B}, H={H} not divisible by {world} ranks")


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from gdn2_package import _lib, gdn2_fwd, gdn2_pipeline
    from gdn2_package.synthetic import make_inputs_torch

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["B"] = args.batch
    B, H = _shard(cfg, world, rank, args.scaling)
    T, D, BT = cfg["T"], cfg["D"], cfg["BT"]
    gdn2_fwd.BT, gdn2_fwd.BC, gdn2_fwd.CLIP = BT, cfg["BC"], cfg["CLIP"]
    cdt = torch.float32 if cfg["dtype"] == "f32" else torch.bfloat16
    names = ("q", "k", "v", "w", "b", "g")
    inp = make_inputs_torch(B, T, H, D, seed=rank, device=dev, h0_std=cfg["h0"], grads=cfg["bwd"])
    devt = {n: inp[n].to(cdt) for n in names}
    extra = [n for n in ("h0", "dout", "dh_final") if n in inp]
    devt.update({n: inp[n] for n in extra})
    del inp
    scale = D ** -0.5

    # --segments: the chunk-parallel scan of gdn2_package.segmented (every
    # sequence cut into S time segments joined by their affine maps); 0 plans S
    from gdn2_package import segmented as SG
    S = args.segments
    if S == 0:
        S = SG.plan_segments(B, T, H, BT, torch.cuda.get_device_properties(dev).multi_processor_count)
    if S > 1 and not (cfg["bwd"] and BT == 128 and D == 128):
        raise SystemExit("--segments needs a fwd+bwd configuration with BT = D = 128")

    def step(d):
        h0 = d.get("h0")
        if S > 1:
            x = [d[n] for n in names]
            r = SG.segmented_forward(*x, scale, h0, S)
            grads = SG.segmented_backward(r[2], d["dout"], d["dh_final"]) if r else None
            if grads is None:   # a sanitiser acted: the serial path
                (o, h), res = gdn2_pipeline._gdn2_core_fwd(*x, scale, h0)
                return o, h, gdn2_pipeline._gdn2_core_bwd(scale, res, (d["dout"], d["dh_final"]))
            return r[0], r[1], grads
        if not cfg["bwd"]:
            p = gdn2_fwd._Prepared(*[d[n] for n in names], scale, h0)
            o, h, _ = gdn2_fwd._run_forward(p)
            return o, h, ()
        (o, h), res = gdn2_pipeline._gdn2_core_fwd(*[d[n] for n in names], scale, h0)
        grads = gdn2_pipeline._gdn2_core_bwd(scale, res, (d["dout"], d["dh_final"]))
        return o, h, grads

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(devt)
    barrier()

    # ---- device-resident timed region (inputs in HBM, larger than L2)
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

    # ---- end-to-end through the public API with host buffers: gdn2_fwd_bwd
    # streams batch shards (copy in, kernels, copy out overlapped)
    from gdn2_package import gdn2_fwd_bwd
    out_host = None
    host = None
    e2e_ms, d2h, h2d = float("nan"), 0, 0

    def e2e_step():
        nonlocal out_host
        o, h, grads = gdn2_fwd_bwd(*[host[n] for n in names], scale, host.get("dout"),
                                   host.get("dh_final"), host.get("h0"), out=out_host)
        outs = [o, h, *(grads or ())]
        if out_host is None:
            out_host = outs
        return outs

    if not args.skip_e2e:
        host = {n: t.cpu().pin_memory() for n, t in devt.items()}
        del devt
        torch.cuda.empty_cache()
        h2d = sum(t.numel() * t.element_size() for t in host.values())
        outs = e2e_step()
        torch.cuda.synchronize()
        d2h = sum(t.numel() * t.element_size() for t in outs)
        del outs
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
    s_in = 4 if cfg["dtype"] == "f32" else 2
    fl, by = flops_per_chunk(BT, D), bytes_per_chunk(BT, D, s_in)
    hbm, bf16, kind = _peaks()
    tpeak, tpeak_kind = tensor_peak(cfg, bf16)
    per_kernel = {}
    for s, (tot, cnt) in prof.items():
        if cnt:
            avg = tot / cnt
            per_kernel[s] = {"avg_ms": avg, "launches": cnt,
                             "tflops": fl[s] * nchunks / (avg * 1e-3) / 1e12,
                             "gbs": by[s] * nchunks / (avg * 1e-3) / 1e9}
            per_kernel[s]["hbm_frac"] = per_kernel[s]["gbs"] / hbm
            per_kernel[s]["tensor_frac"] = per_kernel[s]["tflops"] / tpeak
    top = max(per_kernel, key=lambda s: per_kernel[s]["avg_ms"] * per_kernel[s]["launches"])
    tk = per_kernel[top]
    traffic = NCU_TRAFFIC_PER_CHUNK.get(top) if args.config == 1 else None
    # The bound is the roof the kernel is nearest to; both fractions stay
    # far below 1 for the kernels here, which are latency bound (warp stalls
    # on global loads and barriers, one CTA per SM).
    bound = "hbm" if tk["hbm_frac"] >= tk["tensor_frac"] else "tensor"
    roofline = {
        "kernel": top, "bound": bound,
        "achieved": tk["gbs"] if bound == "hbm" else tk["tflops"],
        "peak": hbm if bound == "hbm" else tpeak,
        "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
        "frac": tk["hbm_frac"] if bound == "hbm" else tk["tensor_frac"],
        "traffic": traffic * nchunks if traffic else None,
        "algorithmic_bytes": by[top] * nchunks,
        "peak_kind": f"{kind} copy bandwidth" if bound == "hbm" else f"{kind}: {tpeak_kind}",
        "limiter": "latency: both fractions well below 1 (see profiles/)",
        "hbm_frac": tk["hbm_frac"],
        "tensor_achieved_tflops": tk["tflops"], "tensor_peak_tflops": tpeak,
        "tensor_peak_kind": f"{kind}: {tpeak_kind}", "tensor_frac": tk["tensor_frac"],
    }
    wf, wb = step_work(dict(cfg, B=B * world, H=H))
    step_roof = {"flops": wf, "bytes": wb,
                 "tflops": wf / (ms_step * 1e-3) / 1e12 / world,
                 "gbs": wb / (ms_step * 1e-3) / 1e9 / world}
    step_roof["tensor_frac"] = step_roof["tflops"] / tpeak
    step_roof["hbm_frac"] = step_roof["gbs"] / hbm
    step_roof["note"] = ("whole step per GPU: spec FLOPs and compulsory bytes / ms_per_step, "
                         "against the same peaks")
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        slices, threads = _cpu_plan(cfg)
        cinp = _cpu_inputs(cfg, slices)
        dt = _cpu_run(cfg, cinp, threads)
        cpu = {"value": slices * T / dt, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": _cpu_sample_text(cfg, slices, threads, dt)}
    line = {
        "metric": METRIC if args.config == 1 else metric_of(cfg),
        "value": tokens / (ms_step * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": args.scaling if world > 1 else "weak",
        "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic (reference distributions, seeded, drawn on the device); inputs "
                "in HBM, larger than L2",
        "config": {"workload": workload_of(cfg, args.config,
                                           f" per GPU (B{B} H{H})" if world > 1 else ""),
                   "global_batch": B * world if H == cfg["H"] else B, "seq_len": T,
                   "heads": H, "head_dim": D,
                   "parallelism": f"dp{world} (batch x head shards, no collective)",
                   "segments": S,
                   "l2": "inputs larger than L2"},
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": sum(v["launches"] for v in per_kernel.values()),
        "roofline": roofline,
        "step_roofline": step_roof,
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
    ap.add_argument("--config", type=int, default=1, choices=[1, 2, 3, 4],
                    help="BASELINE.json configuration (1 = the headline B8 T8192 H6 D128)")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="N>1: weak = every rank runs the whole configuration; strong = its "
                         "(batch, head) units are split over the ranks")
    ap.add_argument("--batch", type=int, default=0,
                    help="override B (profiling of smaller cases only)")
    ap.add_argument("--skip-e2e", action="store_true", help="profiling: skip the host-buffer leg")
    ap.add_argument("--segments", type=int, default=1,
                    help="time segments per sequence for the chunk-parallel scan on one GPU "
                         "(1 = serial scan, 0 = planned for this GPU; fwd+bwd, BT = D = 128)")
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
