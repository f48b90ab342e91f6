"""Benchmark of the Chelis B200 backend (one JSON line on rank 0).

Headline workload: the pre-LN transformer block, forward
and reverse mode, f32 -- batch 8, sequence 2048, d_model 1024, 16 heads of
64, causal softmax attention, GELU MLP 1024 -> 4096 -> 1024, weights
Xavier-uniform and activations N(0, 1) from seed 3 -- data-parallel over
the batch: with --gpus N the global batch of 8 is split across the N ranks
(strong scaling) and the weight gradients (12.6 M f32, 50.3 MB) are summed
across ranks by the library's NCCL communicator every step, each gradient
as soon as the reverse pass has written it, overlapped with the rest of the
pass (chelis_cuda_block_step_dp).  Metric: samples per second of the whole
job.

  value     device-resident inputs, CUDA-event timed over exactly --steps
            steps after --warmup untimed ones, max over ranks.  The working
            set (weights, gradients and the per-rank activations) exceeds the
            126 MB L2, so no flush is needed.
  e2e       the same step from pinned host buffers: this rank's x and dy
            copied to the device, the block step, the all-reduce, and the
            reduced gradients plus dx copied back, inside every timed step;
            as in a training loop the next step's upload and the previous
            step's download run on copy streams while a step computes.
  roofline  the phase group that takes the most time in the step (the
            library's phase timer: CUDA events inside chelis_cuda_block_step),
            its algorithmic FLOPs (useful f32 FLOPs; each runs as 3 tf32 MMA
            terms) over its measured time, against the measured tf32 tensor
            peak / 3 (cuBLAS TF32 GEMM timed in this run).
  cpu_baseline  the oracle (the reference C lane's algorithm restated in C,
            -O2 -ffp-contract=off, OpenMP on every host core) on one sample
            of the batch.
  extra     the other configurations: f32 / f64 GEMM sweeps with pipe
            fractions, the fused chain (config 3), the fused groups, the MLP
            step (config 1), the covariance vmap (config 5), the batched
            GEMM (2b), each with a roofline and, at one GPU, a CPU baseline.

`--impl reference` times the reference C lane's algorithm (the oracle) on
the same workload, one sample of the batch per step, with every host core.
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
sys.path.insert(0, ROOT)

PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_PATH = os.path.join(ROOT, "profiles", "traffic.json")
METRIC = "block_fwd_bwd_samples_per_s"
UNIT = "samples/s"
GLOBAL_BATCH = 8
DATA = "synthetic (Xavier-uniform weights, N(0,1) activations and cotangent, seed 3)"


def load_peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return dict(hbm=float(p["hbm_gbs"]), bf16=float(p["bf16_tflops"]),
                    bf16_sustained=float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                    source="measured")
    except Exception:
        return dict(hbm=6650.0, bf16=1590.0, bf16_sustained=1400.0, source="fallback")


def load_traffic(name):
    try:
        with open(TRAFFIC_PATH) as f:
            return json.load(f).get(name)
    except Exception:
        return None


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def use_all_host_cores():
    """OpenMP threads for the oracle: every host core this process may use
    (set outright: torchrun sets OMP_NUM_THREADS=1 for its ranks)."""
    n = host_cores()
    os.environ["OMP_NUM_THREADS"] = str(n)
    return n


def block_config(world):
    """The workload description both arms print (identical dicts)."""
    return {"workload": "config 4: transformer block fwd+bwd f32 (pre-LN, causal softmax "
                        "attention, GELU MLP), data-parallel over the batch",
            "global_batch": GLOBAL_BATCH, "seq_len": 2048, "d_model": 1024, "heads": 16,
            "head_dim": 64, "d_ff": 4096, "parallelism": f"dp{world}",
            "l2": "working set > 126 MB L2 (weights + gradients 100.6 MB + activations), no flush"}


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during a timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- helpers

def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x, world):
    import torch
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_region(fn, steps, world):
    """CUDA-event time of `steps` calls of fn on the current stream (ms),
    bracketed by barrier + synchronize; max over ranks."""
    import torch
    barrier(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    stop.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(start.elapsed_time(stop), world)


def warm_until_sampling(step, clk, world, limit_s=5.0):
    """Run untimed steps until the clock sampler of every rank has reported
    (or limit_s has passed on every rank).  The stop decision is a MIN
    all-reduce over the ranks after each step, so every rank runs the same
    number of steps."""
    import torch
    t0 = time.time()
    while True:
        step()
        torch.cuda.synchronize()
        done = 1.0 if (clk.lines or time.time() - t0 > limit_s) else 0.0
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([done], dtype=torch.float32, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            done = float(t.item())
        if done:
            return


def timed(fn, steps, warm=3):
    for _ in range(warm):
        fn()
    return time_region(fn, steps, 1) / steps


def measure_pipe_peaks():
    """Denominators for the tensor and FP64 pipes, measured in this run with
    cuBLAS through torch (8192^3, best of a few): tf32 tensor GEMM, f64 GEMM
    (DMMA), and f32 GEMM with tf32 off."""
    import torch
    n = 8192
    out = {}
    g = torch.Generator(device="cuda").manual_seed(0)
    for name, dt, tf32, reps in (("tf32_tflops", torch.float32, True, 5),
                                 ("fp32_tflops", torch.float32, False, 3),
                                 ("fp64_tflops", torch.float64, False, 3)):
        a = torch.rand((n, n), generator=g, device="cuda", dtype=dt)
        b = torch.rand((n, n), generator=g, device="cuda", dtype=dt)
        old = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = tf32
        try:
            for _ in range(2):
                torch.matmul(a, b)
            best = None
            for _ in range(reps):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                torch.matmul(a, b)
                e.record()
                torch.cuda.synchronize()
                ms = s.elapsed_time(e)
                best = ms if best is None else min(best, ms)
        finally:
            torch.backends.cuda.matmul.allow_tf32 = old
        out[name] = round(2 * n ** 3 / best / 1e9, 1)
        del a, b
    torch.cuda.empty_cache()
    out["how"] = "cuBLAS via torch.matmul 8192^3, best of 3-5 (CUDA events), this run"
    return out


# ---------------------------------------------------------------- config 4 (headline)

def block_flops(local_batch, S=2048, D=1024, H=16, F=4096):
    """Useful FLOPs of one block step (forward + VJP) on `local_batch`
    samples, by phase group: matmuls 3 x (2 S D (4D + 2F)) per sample; causal
    attention 2 S^2 D forward, 4 S^2 D reverse."""
    Dh = D // H
    gemm = 3 * 2 * local_batch * S * D * (4 * D + 2 * F)
    att_f = local_batch * H * 2 * S * S * Dh
    att_b = local_batch * H * 4 * S * S * Dh
    return {"gemm": gemm, "attention_fwd": att_f, "attention_bwd": att_b,
            "total": gemm + att_f + att_b}


def phase_group(name):
    if name.startswith("gemm"):
        return "gemm"
    if name.startswith("attention"):
        return name
    return "rows"


def block_phases(step, steps=3):
    """Per-phase ms of the block step (library phase timer), mean of `steps`."""
    import ctypes
    from chelis_b200 import lib as L
    lib = L.load()
    L.call("chelis_cuda_block_timing", 1)
    acc = [0.0] * 16
    try:
        for _ in range(steps):
            step()
            ms = (ctypes.c_float * 16)()
            L.call("chelis_cuda_block_phase_ms", ms, 16)
            for i in range(16):
                acc[i] += ms[i] / steps
    finally:
        L.call("chelis_cuda_block_timing", 0)
    names = [lib.chelis_cuda_block_phase_name(i).decode() for i in range(16)]
    phases = {n: round(v, 4) for n, v in zip(names, acc)}
    groups = {}
    for n, v in zip(names, acc):
        g = phase_group(n)
        groups[g] = round(groups.get(g, 0.0) + v, 4)
    return phases, groups


def bench_block_headline(args, world, rank, peaks, pipes):
    import torch
    from chelis_b200 import dp, ops, workloads as W
    shape = dict(W.BLOCK_SHAPE)
    heads = shape["heads"]
    a, b = dp.shard(GLOBAL_BATCH, world, rank)
    local = b - a
    x_all, dy_all, w = W.torch_block_inputs(seed=3, **shape)
    x = x_all[a:b].contiguous()
    dy = dy_all[a:b].contiguous()
    del x_all, dy_all
    names = list(ops.BLOCK_WEIGHTS)
    grads = dp.FlatGrads({"d" + k: tuple(w[k].shape) for k in names}, "cuda")
    res = {"y": torch.empty_like(x), "dx": torch.empty_like(x)}
    res.update({k: grads[k] for k in grads.views})
    ws = ops.block_workspace(x, w, heads)

    def step():
        # each weight gradient is summed across the ranks as soon as the
        # reverse pass has written it, overlapped with the rest of the pass
        ops.block_step(x, w, heads, 1e-5, dy, workspace=ws, out=res, reduce_grads=True)

    for _ in range(args.warmup):
        step()
    ops.device_status()
    with ClockSampler(torch.cuda.current_device()) as clk:
        # the sampler needs ~1 s to start; keep the GPU busy with untimed
        # steps until every rank's sampler reports (a collective decision, so
        # all ranks run the same number of steps and collectives), then time
        # exactly args.steps
        warm_until_sampling(step, clk, world)
        l0 = ops.launch_count()
        ms = time_region(step, args.steps, world)
        launches = ops.launch_count() - l0
    ops.device_status()
    ms_step = ms / args.steps
    value = GLOBAL_BATCH * args.steps / (ms * 1e-3)

    # where the step's time goes (phase timer; compute only) and the
    # gradient all-reduce alone
    phases, groups = block_phases(lambda: ops.block_step(x, w, heads, 1e-5, dy, workspace=ws,
                                                         out=res))
    ar_ms = serial_ms = 0.0
    if world > 1:
        for _ in range(3):
            dp.allreduce_sum(grads.flat, world)
        ar_ms = time_region(lambda: dp.allreduce_sum(grads.flat, world), 10, world) / 10

        def serial_step():
            ops.block_step(x, w, heads, 1e-5, dy, workspace=ws, out=res)
            dp.allreduce_sum(grads.flat, world)

        for _ in range(2):
            serial_step()
        serial_ms = time_region(serial_step, 5, world) / 5
    fl = block_flops(local)
    dom = max(("gemm", "attention_fwd", "attention_bwd"), key=lambda g: groups.get(g, 0.0))
    dom_ms = groups[dom]
    achieved = fl[dom] / (dom_ms * 1e-3) / 1e12
    f32_peak = pipes["tf32_tflops"] / 3.0
    roofline = {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(f32_peak, 2),
                "unit": "TFLOP/s", "frac": round(achieved / f32_peak, 4),
                "traffic": load_traffic("block_" + dom),
                "kernel": {"gemm": "tf32x3 matmuls of the step (split pre-pass + "
                                   "tf32x3::gemm_pair_kernel, tcgen05 cta_group::2)",
                           "attention_fwd": "attn::fwd_kernel (tcgen05, scores in TMEM)",
                           "attention_bwd": "attn::dkv_kernel + attn::dq_kernel"}[dom],
                "group_ms_per_step": dom_ms, "algorithmic_flop_per_step": fl[dom],
                "peak_source": "measured cuBLAS TF32 GEMM in this run / 3 (an f32 product "
                               "term is 3 tf32 MMA terms)"}
    step_frac = fl["total"] / (ms_step * 1e-3) / 1e12 / f32_peak

    # e2e: pinned host buffers every step.  As a training loop feeds the
    # device: step i+1's x and dy upload on one copy stream and step i's
    # reduced gradients and dx download on another while step i computes
    # (two device buffer sets).  Every step's copies are inside the timed
    # region: the first upload is issued after the start event and the end
    # waits for the last download.
    hx = x.cpu().pin_memory()
    hdy = dy.cpu().pin_memory()
    hg = torch.empty(grads.flat.numel(), dtype=torch.float32).pin_memory()
    hdx = torch.empty(x.shape, dtype=torch.float32).pin_memory()
    xd = [torch.empty_like(x) for _ in range(2)]
    dyd = [torch.empty_like(dy) for _ in range(2)]
    gsets = [grads, dp.FlatGrads({"d" + k: tuple(w[k].shape) for k in names}, "cuda")]
    rsets = []
    for g in gsets:
        r = {"y": torch.empty_like(x), "dx": torch.empty_like(x)}
        r.update({k: g[k] for k in g.views})
        rsets.append(r)
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    fetched = [torch.cuda.Event() for _ in range(2)]

    def upload(b):
        with torch.cuda.stream(up):
            xd[b].copy_(hx, non_blocking=True)
            dyd[b].copy_(hdy, non_blocking=True)
            uploaded[b].record(up)

    def e2e_run(n):
        up.wait_stream(comp)
        upload(0)
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                up.wait_event(computed[1 - b])  # step i-1 is done with set 1 - b
                upload(1 - b)
            comp.wait_event(uploaded[b])
            comp.wait_event(fetched[b])  # step i-2's results are on the host
            ops.block_step(xd[b], w, heads, 1e-5, dyd[b], workspace=ws, out=rsets[b],
                           reduce_grads=True)
            computed[b].record(comp)
            down.wait_event(computed[b])
            with torch.cuda.stream(down):
                hg.copy_(gsets[b].flat, non_blocking=True)
                hdx.copy_(rsets[b]["dx"], non_blocking=True)
                fetched[b].record(down)
        comp.wait_event(fetched[(n - 1) % 2])

    e2e_run(2)
    torch.cuda.synchronize()
    e_steps = max(4, args.steps // 2)
    ems = time_region(lambda: e2e_run(e_steps), 1, world)
    e2e = {"value": round(GLOBAL_BATCH * e_steps / (ems * 1e-3), 2), "unit": UNIT,
           "h2d_bytes_per_step": 2 * x.numel() * 4,
           "d2h_bytes_per_step": grads.flat.numel() * 4 + x.numel() * 4,
           "what": "per rank: x and dy shard H2D; block step; gradient all-reduce; reduced "
                   "gradients and dx D2H; the next step's upload and the previous step's "
                   "download overlap the step on two copy streams"}
    return dict(value=value, ms_per_step=ms_step, launches=launches, clocks=clk.summary(),
                roofline=roofline, e2e=e2e,
                breakdown={"phase_ms": phases, "group_ms": groups,
                           "compute_ms": round(sum(groups.values()), 4),
                           "allreduce_alone_ms": round(ar_ms, 4),
                           "allreduce_overlapped": world > 1,
                           "step_ms_allreduce_after_step": round(serial_ms, 4),
                           "allreduce_mb": round(grads.flat.numel() * 4 / 1e6, 1),
                           "per_rank_batch": local,
                           "step_useful_tflops": round(fl["total"] / (ms_step * 1e-3) / 1e12, 1),
                           "step_frac_of_f32_tensor_peak": round(step_frac, 4)})


def cpu_block_sample():
    """Oracle block step (forward + VJP) on one sample; (samples/s, s, cores)."""
    import numpy as np
    from chelis_b200 import workloads as W
    cores = use_all_host_cores()
    from oracle import oracle as O
    O.lib()
    shape = dict(W.BLOCK_SHAPE, batch=1)
    x, dy, w = W.block_inputs(seed=3, **shape)
    t0 = time.perf_counter()
    O.block_step(x, w, shape["heads"], np.float32(1e-5), dy)
    dt = time.perf_counter() - t0
    return 1.0 / dt, dt, cores


# ---------------------------------------------------------------- extras

def cpu_gemm_sample(n, budget_s, seed=1):
    """Oracle on a bounded sample of output rows of the n^3 f32 product;
    returns (TFLOP/s, rows, seconds, threads)."""
    import numpy as np
    from chelis_b200 import workloads as W
    threads = use_all_host_cores()
    from oracle import oracle as O
    a, b = W.gemm_inputs(n, n, n, np.float32, seed=seed)
    O.lib()
    t0 = time.perf_counter()
    O.gemm(a[:threads], b)
    dt = time.perf_counter() - t0
    per_row = dt / threads
    rows = int(max(threads, min(n, budget_s / max(per_row, 1e-9))))
    rows = (rows // threads) * threads or threads
    t0 = time.perf_counter()
    O.gemm(a[:rows], b)
    dt = time.perf_counter() - t0
    return 2.0 * rows * n * n / dt / 1e12, rows, dt, threads


def bench_gemm(args, peaks, pipes, with_cpu):
    """Config 2: the f32 sweep (3xTF32) incl. 8192^3 with its main-kernel
    roofline and host-buffer e2e, and the f64 sweep (DMMA)."""
    import torch
    from chelis_b200 import lib as L
    from chelis_b200 import ops, workloads as W
    out = {}
    f32_peak = pipes["tf32_tflops"] / 3.0
    sweep = {}
    for n in (512, 1024, 2048, 4096, 8192):
        a, b = W.torch_gemm_inputs(n, n, n, torch.float32, seed=1)
        c = torch.empty((n, n), dtype=torch.float32, device="cuda")
        ms = timed(lambda: ops.matmul(a, b, out=c), 20 if n < 8192 else 10)
        t = 2 * n ** 3 / ms / 1e9
        sweep[str(n)] = {"tflops": round(t, 2), "ms": round(ms, 4),
                         "frac_f32_tensor_peak": round(t / f32_peak, 4)}
    out["gemm_f32_sweep"] = sweep
    n = 8192
    # roofline of the main kernel alone on pre-split operands
    kp = (n + 31) // 32 * 32
    ahi = torch.empty((n, kp), dtype=torch.float32, device="cuda")
    alo, bhi, blo = torch.empty_like(ahi), torch.empty_like(ahi), torch.empty_like(ahi)
    ops._prepare(a)
    L.call("chelis_cuda_tf32x3_split", 0, 0, n, n, a.data_ptr(), n, 0, 1, ahi.data_ptr(), alo.data_ptr())
    L.call("chelis_cuda_tf32x3_split", 1, 1, n, n, b.data_ptr(), n, 0, 1, bhi.data_ptr(), blo.data_ptr())

    def main_only():
        L.call("chelis_cuda_sgemm_tf32x3_presplit", n, n, n, 1, 0, ahi.data_ptr(), alo.data_ptr(),
               1, bhi.data_ptr(), blo.data_ptr(), c.data_ptr(), n, 0)

    kms = timed(main_only, 10)
    ach = 2 * n ** 3 / (kms * 1e-3) / 1e12
    del ahi, alo, bhi, blo
    ha, hb = a.cpu().pin_memory(), b.cpu().pin_memory()
    hc = torch.empty((n, n), dtype=torch.float32).pin_memory()
    ems = timed(lambda: ops.matmul_host(ha, hb, out=hc), 3, 1)
    out["gemm_f32_8192"] = {
        "tflops": sweep["8192"]["tflops"], "ms": sweep["8192"]["ms"],
        "roofline": {"bound": "tensor", "achieved": round(ach, 2), "peak": round(f32_peak, 2),
                     "unit": "TFLOP/s", "frac": round(ach / f32_peak, 4),
                     "traffic": load_traffic("gemm_tf32x3_8192"), "kernel_ms": round(kms, 4),
                     "kernel": "tf32x3::gemm_pair_kernel (tcgen05 cta_group::2 kind::tf32)",
                     "peak_source": "measured cuBLAS TF32 / 3"},
        "e2e": {"value": round(2 * n ** 3 / ems / 1e9, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": 2 * n * n * 4, "d2h_bytes_per_step": n * n * 4}}
    del a, b, c, ha, hb, hc
    torch.cuda.empty_cache()
    if with_cpu:
        v, rows, dt, threads = cpu_gemm_sample(n, 8.0)
        out["gemm_f32_8192"]["cpu_baseline"] = {
            "value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of {n} output rows of the {n}^3 f32 product ({dt:.1f} s)"}
    f64 = {}
    for n in (512, 1024, 2048, 4096, 8192):
        a, b = W.torch_gemm_inputs(n, n, n, torch.float64, seed=1)
        c = torch.empty((n, n), dtype=torch.float64, device="cuda")
        ms = timed(lambda: ops.matmul(a, b, out=c), 10 if n < 8192 else 3, 2)
        t = 2 * n ** 3 / ms / 1e9
        f64[str(n)] = {"tflops": round(t, 2), "ms": round(ms, 4),
                       "frac_fp64_peak": round(t / pipes["fp64_tflops"], 4)}
        del a, b, c
    out["gemm_f64_sweep"] = dict(f64, peak_source="measured cuBLAS DGEMM 8192^3 in this run",
                                 kernel="dmma::dgemm_async_kernel (mma.sync m16n8k4 f64)")
    torch.cuda.empty_cache()
    return out


def bench_rows(args, peaks, with_cpu):
    """Config 3 (fused chain fwd / adjoint), the fused groups alone and
    generic FusedElem groups on [16384, 4096] f32; config 1 (MLP step)."""
    import numpy as np
    import torch
    from chelis_b200 import ops, workloads as W
    out = {}
    hbm = peaks["hbm"]
    x, g, be = W.torch_chain_inputs()
    rows, hidden = x.shape
    state = {}

    def fwd():
        state["rs"], state["saved"] = ops.chain_fwd_save(x, g, be, 1e-5, 42, 0.1)

    fms = timed(fwd, 10)
    bms = timed(lambda: ops.chain_bwd_saved(x, g, be, 1e-5, 0.1, state["saved"]), 10)
    saved = state["saved"].numel() * 4
    # algorithmic bytes: X read + gamma, beta + row sums (forward); X read, dX
    # written, dgamma / dbeta (adjoint); the saved state both ways
    fbytes = rows * hidden * 4 + 2 * hidden * 4 + rows * 4 + saved
    bbytes = 2 * rows * hidden * 4 + 4 * hidden * 4 + saved
    chain = {"fwd": {"gbs": round(fbytes / fms / 1e6, 1), "ms": round(fms, 4),
                     "roofline": {"bound": "hbm", "achieved": round(fbytes / fms / 1e6, 1),
                                  "peak": hbm, "unit": "GB/s",
                                  "frac": round(fbytes / fms / 1e6 / hbm, 4),
                                  "traffic": load_traffic("chain_fwd_16384x4096")}},
             "bwd": {"gbs": round(bbytes / bms / 1e6, 1), "ms": round(bms, 4),
                     "roofline": {"bound": "hbm", "achieved": round(bbytes / bms / 1e6, 1),
                                  "peak": hbm, "unit": "GB/s",
                                  "frac": round(bbytes / bms / 1e6 / hbm, 4),
                                  "traffic": load_traffic("chain_bwd_16384x4096")}}}
    if with_cpu:
        cores = use_all_host_cores()
        from oracle import oracle as O
        O.lib()
        xs, gs, bs = (np.ascontiguousarray(t[:512].cpu().numpy()) if t.dim() == 2 else
                      t.cpu().numpy() for t in (x, g, be))
        t0 = time.perf_counter()
        O.chain_fwd(xs, gs, bs, np.float32(1e-5), 42, np.float32(0.1))
        dt = time.perf_counter() - t0
        sb = 512 * hidden * 4 + 2 * hidden * 4 + 512 * 4
        chain["fwd"]["cpu_baseline"] = {"value": round(sb / dt / 1e9, 3), "unit": "GB/s",
                                        "cores": cores, "kind": "port",
                                        "sample": f"512 of {rows} rows ({dt:.2f} s)"}
        t0 = time.perf_counter()
        O.chain_bwd(xs, gs, bs, np.float32(1e-5), 42, np.float32(0.1))
        dt = time.perf_counter() - t0
        sb = 2 * 512 * hidden * 4 + 4 * hidden * 4
        chain["bwd"]["cpu_baseline"] = {"value": round(sb / dt / 1e9, 3), "unit": "GB/s",
                                        "cores": cores, "kind": "port",
                                        "sample": f"512 of {rows} rows ({dt:.2f} s)"}
    out["chain_16384x4096"] = chain
    y = torch.softmax(x, -1)
    nb = rows * hidden * 4
    groups = {
        "layer_norm": (lambda: ops.layer_norm(x, g, be, 1e-5), 2 * nb),
        "softmax": (lambda: ops.softmax_rows(x), 2 * nb),
        "softmax_bwd": (lambda: ops.softmax_rows_bwd(y, x), 3 * nb),
        "row_sum": (lambda: ops.row_sum(x), nb + rows * 4),
        "col_sum": (lambda: ops.col_sum(x), nb + hidden * 4),
        "row_max": (lambda: ops.row_max(x), nb + rows * 4),
        "dropout": (lambda: ops.dropout(x, 42, 0.1), 2 * nb),
    }
    fused = {}
    for name, (fn, nbytes) in groups.items():
        ms_g = timed(fn, 10)
        fused[name] = {"ms": round(ms_g, 4), "gbs": round(nbytes / ms_g / 1e6, 1),
                       "frac_hbm": round(nbytes / ms_g / 1e6 / hbm, 3)}
    out["fused_groups_16384x4096"] = fused
    from chelis_b200 import fused as F
    consts = [torch.tensor(v, device="cuda") for v in (0.044715, 0.7978845608, 0.5, 1.0)]
    gelu = ("mul x0 x0; mul v0 x0; mul v1 x1; add v2 x0; mul v3 x2; tanh v4; "
            "add v5 x4; mul v6 x0; mul v7 x3")
    flat = x.reshape(-1)
    elem = {
        "affine": (lambda c=F.parse("mul x0 x1; add v0 x2"): ops.fused_elementwise(c, [x, g, be]),
                   2 * nb),
        "exp": (lambda c=F.parse("exp x0"): ops.fused_elementwise(c, [x]), 2 * nb),
        "gelu": (lambda c=F.parse(gelu): ops.fused_elementwise(c, [x, *consts]), 2 * nb),
        "sum_sq_rows": (lambda c=F.parse("mul x0 x0"): ops.fused_reduce(c, [x], axis=1),
                        nb + rows * 4),
        "sum_sq_cols": (lambda c=F.parse("mul x0 x0"): ops.fused_reduce(c, [x], axis=0),
                        nb + hidden * 4),
        "max_abs_rows": (lambda c=F.parse("abs x0"): ops.fused_reduce(c, [x], axis=1, kind="max"),
                         nb + rows * 4),
        "sum_sq_all": (lambda c=F.parse("mul x0 x0"): ops.fused_reduce(c, [flat], axis=0), nb + 4),
    }
    generic = {}
    for name, (fn, nbytes) in elem.items():
        ms_g = timed(fn, 10)
        generic[name] = {"ms": round(ms_g, 4), "gbs": round(nbytes / ms_g / 1e6, 1),
                         "frac_hbm": round(nbytes / ms_g / 1e6 / hbm, 3)}
    out["fused_elem_16384x4096"] = generic
    del x, g, be, state, y, flat
    # config 1: MLP step (latency-bound: 1.05e8 FLOP in a handful of launches)
    x, labels, w1, b1, w2, b2 = W.torch_mlp_inputs()
    l0 = ops.launch_count()
    ops.mlp_step(x, labels, w1, b1, w2, b2)
    launches = ops.launch_count() - l0
    ms = timed(lambda: ops.mlp_step(x, labels, w1, b1, w2, b2), 50)
    flop = 2 * 128 * (784 * 256 + 256 * 10) + 2 * 128 * (784 * 256 + 2 * 256 * 10)
    mlp = {"us_per_step": round(ms * 1e3, 1), "launches_per_step": launches,
           "roofline": {"bound": "latency", "achieved": round(flop / (ms * 1e-3) / 1e12, 3),
                        "unit": "TFLOP/s", "flop_per_step": flop,
                        "note": "1.05e8 FLOP over launches_per_step dependent kernels; repeated "
                                "calls replay them as one captured CUDA graph"}}
    if with_cpu:
        cores = use_all_host_cores()
        from oracle import oracle as O
        xs, ls, a1, c1, a2, c2 = (t.cpu().numpy() for t in (x, labels, w1, b1, w2, b2))
        O.mlp_step(xs, ls, a1, c1, a2, c2)
        t0 = time.perf_counter()
        reps = 5
        for _ in range(reps):
            O.mlp_step(xs, ls, a1, c1, a2, c2)
        dt = (time.perf_counter() - t0) / reps
        mlp["cpu_baseline"] = {"value": round(dt * 1e6, 1), "unit": "us/step", "cores": cores,
                               "kind": "port", "sample": f"the full step, mean of {reps}"}
    out["mlp_step"] = mlp
    return out


def bench_sharded(args, world, rank, peaks, pipes, with_cpu):
    """Configs that shard across GPUs, at every N (max over ranks): config 4
    weak (8 samples per rank), config 5 and the batched GEMM of config 2
    along their vmap axis (no collective)."""
    import numpy as np
    import torch
    from chelis_b200 import dp, ops, workloads as W
    out = {}
    shape = dict(W.BLOCK_SHAPE)
    S, D, F = shape["seq"], shape["d_model"], shape["d_ff"]
    per_sample = block_flops(1, S, D, shape["heads"], F)["total"]
    if world > 1:
        x, dy, w = W.torch_block_inputs(seed=3 + rank, **shape)
        names = list(ops.BLOCK_WEIGHTS)
        grads = dp.FlatGrads({"d" + k: tuple(w[k].shape) for k in names}, "cuda")
        res = {"y": torch.empty_like(x), "dx": torch.empty_like(x)}
        res.update({k: grads[k] for k in grads.views})
        ws = ops.block_workspace(x, w, shape["heads"])

        def step():
            ops.block_step(x, w, shape["heads"], 1e-5, dy, workspace=ws, out=res)
            dp.allreduce_sum(grads.flat, world)

        for _ in range(3):
            step()
        ms = time_region(step, 5, world) / 5
        out["block_dp_weak"] = {"samples_per_s": round(8 * world / ms * 1e3, 1),
                                "ms_per_step": round(ms, 3), "per_rank_batch": 8,
                                "scaling": "weak (8 samples per rank)",
                                "tflops": round(8 * world * per_sample / ms / 1e9, 1)}
        del x, dy, w, grads, res, ws
        torch.cuda.empty_cache()
    # config 5: covariance / risk, 65536 portfolios split across ranks
    cnt, T, A = (W.PORTFOLIO_SHAPE[k] for k in ("count", "t", "a"))
    lo, hi = dp.shard(cnt, world, rank)
    r, wv = W.torch_portfolio_inputs(count=hi - lo, seed=4 + rank)
    for _ in range(2):
        ops.portfolio(r, wv)
    ms = time_region(lambda: ops.portfolio(r, wv), 3, world) / 3
    flop = cnt * 2.10e6
    nbytes = cnt * (T * A * 8 + A * 8 + A * A * 8 + 8 + T * 8)
    fp64 = flop / ms / 1e9
    gbs = nbytes / ms / 1e6
    port = {"portfolios_per_s": round(cnt / ms * 1e3, 1), "ms": round(ms, 3),
            "fp64_tflops": round(fp64, 2), "scaling": "strong (65536 portfolios)",
            "roofline": {"bound": "fp64", "achieved": round(fp64, 2),
                         "peak": pipes["fp64_tflops"], "unit": "TFLOP/s",
                         "frac": round(fp64 / pipes["fp64_tflops"], 4),
                         "hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / peaks["hbm"], 4),
                         "traffic": load_traffic("portfolio_4096"),
                         "algorithmic": "2.10 MFLOP and 164 KB per portfolio"}}
    if with_cpu and world == 1:
        cores = use_all_host_cores()
        from oracle import oracle as O
        rs, wsn = W.portfolio_inputs(count=512, seed=4)
        O.lib()
        t0 = time.perf_counter()
        O.portfolio(rs, wsn)
        dt = time.perf_counter() - t0
        port["cpu_baseline"] = {"value": round(512 / dt, 1), "unit": "portfolios/s",
                                "cores": cores, "kind": "port",
                                "sample": f"512 of {cnt} portfolios ({dt:.2f} s)"}
    out["portfolio_vmap"] = port
    del r, wv
    # config 2b: 256 x [512 x 512] . [512 x 512] f32, batch split across ranks
    lo, hi = dp.shard(256, world, rank)
    A_, B_ = W.torch_gemm_inputs(512, 512, 512, torch.float32, seed=1 + rank, batch=hi - lo)
    C_ = torch.empty((hi - lo, 512, 512), dtype=torch.float32, device="cuda")
    for _ in range(3):
        ops.matmul(A_, B_, out=C_)
    ms = time_region(lambda: ops.matmul(A_, B_, out=C_), 10, world) / 10
    t = 256 * 2 * 512 ** 3 / ms / 1e9
    f32_peak = pipes["tf32_tflops"] / 3.0
    out["gemm_batched_vmap"] = {"tflops": round(t, 2), "ms": round(ms, 3),
                                "scaling": "strong (batch 256)",
                                "roofline": {"bound": "tensor", "achieved": round(t, 2),
                                             "peak": round(f32_peak, 2), "unit": "TFLOP/s",
                                             "frac": round(t / f32_peak, 4)}}
    del A_, B_, C_
    _ = np
    return out


# ---------------------------------------------------------------- reference arm

def run_reference(args, world, rank):
    """The reference C lane's algorithm (the oracle) on the headline
    workload: each step is the block forward + VJP of one sample of the
    global batch (sample i mod 8), on every host core."""
    if rank != 0:
        return
    import numpy as np
    from chelis_b200 import workloads as W
    cores = use_all_host_cores()
    from oracle import oracle as O
    O.lib()
    shape = dict(W.BLOCK_SHAPE)
    x, dy, w = W.block_inputs(seed=3, **shape)
    times = []
    for i in range(args.warmup + args.steps):
        j = i % GLOBAL_BATCH
        t0 = time.perf_counter()
        O.block_step(x[j:j + 1], w, shape["heads"], np.float32(1e-5), dy[j:j + 1])
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
    per_sample = statistics.median(times)
    value = 1.0 / per_sample
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_sample * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": DATA,
        "config": block_config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": "one sample of the global batch per step (block forward + "
                                   "VJP at S 2048, d 1024), oracle restatement of the C lane"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="chelis", choices=["chelis", "reference"])
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return

    import torch
    world, rank, local = dist_setup(args)
    peaks = load_peaks()
    if world > 1:
        from chelis_b200 import dp
        dp.native_init(world, rank)
    pipes = measure_pipe_peaks()
    res = bench_block_headline(args, world, rank, peaks, pipes)
    with_cpu = rank == 0 and world == 1 and not args.no_cpu
    extras = {}
    if not args.no_extras:
        if world == 1:
            extras.update(bench_gemm(args, peaks, pipes, with_cpu))
            extras.update(bench_rows(args, peaks, with_cpu))
        extras.update(bench_sharded(args, world, rank, peaks, pipes, with_cpu))
    cpu = None
    if with_cpu:
        v, dt, cores = cpu_block_sample()
        cpu = {"value": round(v, 4), "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"one sample of the batch: block forward + VJP at S 2048, d 1024 "
                         f"({dt:.2f} s), oracle restatement of the C lane"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(res["value"], 2), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(res["ms_per_step"], 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": DATA,
            "config": block_config(world),
            "roofline": res["roofline"], "cpu_baseline": cpu, "e2e": res["e2e"],
            "gpu_launches": res["launches"], "clocks": res["clocks"],
            "breakdown": res["breakdown"], "pipe_peaks": pipes,
        }
        if extras:
            line["extra"] = extras
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        from chelis_b200 import dp
        torch.cuda.synchronize()
        dist.barrier()
        dp.native_finalize()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
