#!/usr/bin/env python
"""Benchmark of the B200 SDPA forward -- prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload C3]

Metric (the benchmark baseline's): SDPA forward TFLOP/s (4*B*H*N^2*D FLOPs, halved for causal)
and ms per step, against the measured B200 dense bf16/fp16 tensor peak.  A step is one forward
pass over one batch of seeded synthetic inputs (torch.randn iid N(0,1), the reference's
generator).  Default workload: C3 = B2 H8 N2048 D128 fp16 top-left causal, seed 2.

* ``value``       device time of the kernel alone (CUDA events on the launching stream, one
                  pair per step), inputs resident in HBM, L2 flushed (256 MiB write) before
                  every timed launch; whole-job FLOPs / max-over-ranks time.
* ``e2e``         the same metric through the public op (torch.ops.fused_attn.forward) with
                  pinned HOST buffers: q/k/v copied in (one copy from one pinned buffer) and
                  O/LSE copied out inside every step; steps double-buffered over three streams
                  (the next step's upload overlaps this step's kernel and download), as a caller
                  streaming batches would run.
* ``roofline``    tensor-bound: achieved TFLOP/s of the kernel / measured bf16 peak
                  (MEASURED_PEAKS.json, burst figure: the kernel is timed alone).  ``traffic``
                  is the per-launch DRAM bytes of the committed ncu summary for this workload.
* ``cpu_baseline`` the reference's own fp64 CPU oracle (oracle/_ref, else the C restatement) on
                  a bounded sample of the workload, on this host's cores (rank 0, N=1 only).

Multi-GPU (``torchrun --nproc-per-node N bench.py --gpus N``): one process per GPU, weak scaling:
rank r runs the same per-GPU workload on its own shard of a global batch of N x B (seed + r), no
collective on the data path; NCCL only reduces the per-rank device time (max) off the hot path.
Every run (N = 1 included) also measures the long-context configuration the way the baseline
names it: C4's 32 heads of one N=16384 sequence split into N contiguous blocks of 32/N heads
(fused_attn.sharding), every rank regenerating the seed-3 tensor and taking its block (strong
scaling, ``secondary.c4_strong``).  After its timing, each rank's LSE and per-head O checksums are
all-gathered and rank 0 compares them with one launch over all 32 heads on its own GPU (the same
kernel on the same inputs: bit-identical).  ``--workload C4`` makes that split the headline.

``--impl reference``: the reference's CPU implementation of the path (its fp64 oracle, which is
the only implementation of the path that runs on this machine class besides ours) on the host
cores, on the same workload/metric, each step a bounded sample (one (b, h) head).  It loads the
workload generator by file path and the reference's compiled oracle, nothing of the fused_attn
package, and reports the same ``config`` as our line.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "fused-attention-cuda_b200"))
WORKLOADS_PY = ROOT / "fused-attention-cuda_b200" / "fused_attn" / "workloads.py"

METRIC = "SDPA fwd ms & TFLOP/s, B2H8N2048 D64/128 fp16, % of B200 tensor peak"
UNIT = "TFLOP/s"
FLUSH_BYTES = 256 << 20  # >= 2x the 126 MB L2
FALLBACK_PEAK_TFLOPS = 1590.0


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def load_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except Exception:
        return FALLBACK_PEAK_TFLOPS, "fallback 1.59 PFLOP/s (MEASURED_PEAKS.json absent)"


def profile_traffic(workload: str) -> int | None:
    """Per-launch DRAM bytes from the committed ncu summary (profiles/), if one exists."""
    for f in sorted((ROOT / "profiles").glob("*.txt")):
        try:
            text = f.read_text()
        except OSError:
            continue
        if f"workload: {workload}" not in text:
            continue
        for line in text.splitlines():
            if line.startswith("dram_bytes_per_launch:"):
                try:
                    return int(float(line.split(":", 1)[1].split()[0]))
                except ValueError:
                    return None
    return None


# ------------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi SM clock / throttle-reason sampler around the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples: list[tuple[float, list[str]]] = []
        self.proc = None
        self.thread = None
        self.t0 = self.t1 = None
        # NVML read every ~2 ms as well: nvidia-smi's 50 ms period can miss a timed region of a
        # few milliseconds entirely.  (t, sm MHz, max sm MHz, clocks-event-reason bit mask)
        self.fast: list[tuple[float, float, float, int]] = []
        self.fast_stop = threading.Event()
        self.fast_thread = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        self.fast_thread = threading.Thread(target=self._poll_nvml, daemon=True)
        self.fast_thread.start()

    def _poll_nvml(self) -> None:
        """Read-only NVML queries of the SM clock and the clocks-event reasons."""
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            while not self.fast_stop.is_set():
                sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                why = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.fast.append((time.time(), sm, mx, why))
                time.sleep(0.002)
            pynvml.nvmlShutdown()
        except Exception:  # NVML absent or refused: the nvidia-smi samples stand alone
            return

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.samples.append((time.time(), [x.strip() for x in line.split(",")]))

    def window(self, t0: float, t1: float) -> None:
        self.t0, self.t1 = t0, t1

    def median_between(self, t0: float, t1: float) -> float | None:
        """Median SM clock (MHz) of the samples taken between t0 and t1 (wall clock), or None."""
        sm = []
        for t, s in list(self.samples):
            if t0 <= t <= t1:
                try:
                    sm.append(float(s[1]))
                except (ValueError, IndexError):
                    continue
        return statistics.median(sm) if sm else None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        self.fast_stop.set()
        if self.fast_thread:
            self.fast_thread.join(timeout=2)
        inside = [s for t, s in self.samples if self.t0 is not None and self.t0 <= t <= self.t1]
        fast_in = [f for f in self.fast if self.t0 is not None and self.t0 <= f[0] <= self.t1]
        if not inside and fast_in:
            bits = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
                    "sw_power_cap": 0x4}
            reasons = sorted(n for n, b in bits.items() if any(f[3] & b for f in fast_in))
            return {"sm_mhz": statistics.median(f[1] for f in fast_in),
                    "sm_max_mhz": max(f[2] for f in fast_in), "reasons": reasons,
                    "samples": len(fast_in), "samples_in_timed_region": len(fast_in),
                    "source": "NVML every ~2 ms (the timed region is shorter than nvidia-smi's "
                              "50 ms period)"}
        use = inside or [s for _, s in self.samples]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in use:
            try:
                sm.append(float(s[1]))
                mx.append(float(s[2]))
            except (ValueError, IndexError):
                continue
            for n, val in zip(names, s[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(use), "samples_in_timed_region": len(inside)}


# ------------------------------------------------------------------------------------------
_WL = None


def workloads():
    """fused_attn/workloads.py (seeded generator, FLOP/byte models, CONFIGS) loaded by file path,
    so that the reference arm does not import the fused_attn package (whose __init__ maps the
    CUDA extension)."""
    global _WL
    if _WL is None:
        import importlib.util

        spec = importlib.util.spec_from_file_location("fa_bench_workloads", WORKLOADS_PY)
        mod = importlib.util.module_from_spec(spec)
        sys.modules["fa_bench_workloads"] = mod  # dataclasses resolve their module by name
        spec.loader.exec_module(mod)
        _WL = mod
    return _WL


def workload_config(name: str):
    key = {"c2": "C2", "c2c": "C2c", "c3": "C3", "c3bf16": "C3bf16", "c4": "C4"}.get(name.lower())
    if key is None:
        raise SystemExit(f"unknown workload {name}")
    return workloads().CONFIGS[key]


def headline_config(base, world: int) -> tuple[dict, object, str]:
    """The JSON line's ``config`` for workload `base` on `world` ranks (both arms print the same),
    the per-rank configuration, and the scaling kind."""
    wl = workloads()
    if base.name == "C4":
        hs = base.H // world
        cfg = wl.Config("C4", base.B, hs, base.N, base.D, base.dtype, base.seed, base.causal)
        scaling, global_batch = "strong", base.B
        parallelism = f"head-sharded x{world} ({hs} heads/GPU), no collective"
        l2 = "flushed before every timed launch (256 MiB write); inputs > L2"
    else:
        cfg = base
        scaling, global_batch = "weak", base.B * world
        parallelism = f"batch-sharded dp{world}, no collective"
        l2 = "flushed before every timed launch (256 MiB write); inputs < L2"
    config = {
        "workload": base.label(),
        "global_batch": global_batch,
        "seq_len": cfg.N,
        "heads_per_gpu": cfg.H,
        "head_dim": cfg.D,
        "causal": cfg.causal,
        "parallelism": parallelism,
        "l2": l2,
        "timing": "CUDA events per launch on the launching stream; max over ranks",
    }
    return config, cfg, scaling


def time_kernel(fn, steps: int, warmup: int, flush, stream) -> list[float]:
    """Per-step device times (ms) of fn() on `stream`, L2 flushed before every launch."""
    import torch

    for _ in range(warmup):
        flush.zero_()
        fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()  # queued first: the GPU is busy while the host enqueues the launch
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def cpu_sample(cfg, budget_s: float, threads: int) -> dict:
    """Times the reference's fp64 oracle on whole (b, h) heads of `cfg` until `budget_s`."""
    import oracle

    attention_flops, make_qkv = workloads().attention_flops, workloads().make_qkv
    kind = "reference" if oracle.ref_available() else "port"
    heads_done, flops, elapsed = 0, 0.0, 0.0
    total_heads = cfg.B * cfg.H
    q, k, v = make_qkv(cfg.B, cfg.H, cfg.N, cfg.D, dtype=cfg.dtype, hkv=cfg.hkv, seed=cfg.seed)
    while heads_done < total_heads and elapsed < budget_s:
        b, h = divmod(heads_done, cfg.H)
        qs, ks, vs = q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1], v[b:b + 1, h:h + 1]
        qs, ks, vs = (t.double().contiguous() for t in (qs, ks, vs))
        t0 = time.perf_counter()
        if kind == "reference":
            _, _, used = oracle.ref_attention(qs, ks, vs, causal=cfg.causal, threads=threads)
        else:
            oracle.attention(qs, ks, vs, causal=cfg.causal, threads=threads)
            used = threads
        elapsed += time.perf_counter() - t0
        flops += attention_flops(1, 1, cfg.N, cfg.D, cfg.causal)
        heads_done += 1
    return {"value": flops / elapsed / 1e12, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{heads_done} of {total_heads} (b,h) heads of {cfg.label()}, fp64, "
                      f"{elapsed:.1f} s, rows split over {threads} threads",
            "ms_per_head": 1e3 * elapsed / max(heads_done, 1)}


# ------------------------------------------------------------------------------------------
def run_reference(args) -> int:
    """--impl reference: the reference's CPU implementation of the path (rank 0 only)."""
    if env_int("RANK", 0) != 0:
        return 0
    sys.path.insert(0, str(ROOT))
    import oracle

    wl = workloads()
    attention_flops, make_qkv = wl.attention_flops, wl.make_qkv
    base = workload_config(args.workload)
    config, _, scaling = headline_config(base, max(1, args.gpus))
    cfg = base
    threads = oracle.default_threads()
    kind = "reference" if oracle.ref_available() else "port"
    q, k, v = make_qkv(cfg.B, cfg.H, cfg.N, cfg.D, dtype=cfg.dtype, hkv=cfg.hkv, seed=cfg.seed)
    heads = [(b, h) for b in range(cfg.B) for h in range(cfg.H)]

    def step(i):
        b, h = heads[i % len(heads)]
        qs, ks, vs = (t[b:b + 1, h:h + 1].double().contiguous() for t in (q, k, v))
        if kind == "reference":
            oracle.ref_attention(qs, ks, vs, causal=cfg.causal, threads=threads)
        else:
            oracle.attention(qs, ks, vs, causal=cfg.causal, threads=threads)

    for i in range(args.warmup):
        step(i)
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        step(args.warmup + i)
        times.append(time.perf_counter() - t0)
    f_step = attention_flops(1, 1, cfg.N, cfg.D, cfg.causal)
    value = f_step * len(times) / sum(times) / 1e12
    dt = {"torch.float16": "fp16", "torch.bfloat16": "bf16"}.get(str(cfg.dtype), "fp32")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * sum(times) / len(times), "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "fp64",
        "data": f"synthetic: torch.randn seed {cfg.seed}, rounded to {dt}, upcast to fp64",
        "config": config,
        "protocol": "host wall clock (perf_counter) per step; one (b, h) head of the workload per "
                    "step (bounded sample), the reference's fp64 oracle on all host threads",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": "one (b, h) head per step, cycling through the heads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args) -> int:
    import torch
    import torch.distributed as dist

    import fused_attn

    wl = workloads()
    attention_bytes, attention_flops, make_qkv = wl.attention_bytes, wl.attention_flops, wl.make_qkv

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.gpus != world and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the kernel has no CPU fallback)")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=dev)
    if not fused_attn.is_available():
        raise SystemExit("fused_attn._C is not built (python fused-attention-cuda_b200/build.py)")

    from fused_attn import sharding

    base = workload_config(args.workload)
    if base.name == "C4" and base.H % world:
        raise SystemExit(f"C4 has {base.H} heads, not divisible by {world}")
    config, cfg, scaling = headline_config(base, world)
    if base.name == "C4":
        # Strong scaling: the 32 heads of one sequence split into contiguous per-rank blocks.
        q_all, k_all, v_all = make_qkv(base.B, base.H, base.N, base.D, dtype=base.dtype,
                                       seed=base.seed)
        q, k, v = (t.to(dev) for t in sharding.shard_heads(q_all, k_all, v_all, world, rank))
        del q_all, k_all, v_all
    else:
        # Weak scaling: same per-GPU workload, rank r owns batch shard r (seed + r).
        q, k, v = make_qkv(cfg.B, cfg.H, cfg.N, cfg.D, dtype=cfg.dtype,
                           seed=sharding.batch_seed(cfg.seed, rank), device=dev)

    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    scale = 1.0 / math.sqrt(cfg.D)
    op = torch.ops.fused_attn.forward

    def fwd():
        return op(q, k, v, cfg.causal, scale)

    o, lse = fwd()
    torch.cuda.synchronize()
    err, bits = fused_attn.last_device_error()
    if err != 0:
        raise SystemExit(f"device status after the first launch: {err} bits={bits:#x}")

    sampler = ClockSampler(local_rank) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(1.0)  # nvidia-smi start-up
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_wall0 = time.time()
    times = time_kernel(fwd, args.steps, args.warmup, flush, stream)
    torch.cuda.synchronize()
    t_wall1 = time.time()
    if world > 1:
        dist.barrier()
    if sampler:
        sampler.window(t_wall0, t_wall1)

    # ---- end to end through the public op, host buffers, copies inside every step -------
    # Every step uploads its q, k, v from pinned host memory, runs fused_attn.forward and
    # downloads O and LSE.  The caller keeps a step's q, k, v in one pinned buffer (the layout a
    # fused QKV projection produces), so the upload is one copy: PCIe sustains ~55 GB/s for one
    # 25 MB copy and ~52 for three 8 MB ones.  Steps are double-buffered over three streams, as a
    # caller streaming independent batches would run them: step i+1's upload (host-to-device copy
    # engine) overlaps step i's kernel and download (device-to-host engine).
    def packed(tensors, **kw):
        """One flat buffer holding `tensors`' shapes back to back (256-byte aligned), and views."""
        el = q.element_size()
        offs, n = [], 0
        for t in tensors:
            offs.append(n)
            n += -(-t.numel() * el // 256) * 256 // el
        flat = torch.empty(n, dtype=q.dtype, **kw)
        return flat, [flat[a:a + t.numel()].view(t.shape) for a, t in zip(offs, tensors)]

    qkv_h, views_h = packed((q, k, v), pin_memory=True)
    for t, src in zip(views_h, (q, k, v)):
        t.copy_(src.cpu())
    oh = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)
    lh = torch.empty(lse.shape, dtype=lse.dtype, pin_memory=True)
    dbuf = [packed((q, k, v), device=dev) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    in_done = [torch.cuda.Event() for _ in range(2)]
    buf_free = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        b = i & 1
        flat_d, (qd, kd, vd) = dbuf[b]
        with torch.cuda.stream(s_in):
            s_in.wait_event(buf_free[b])  # the kernel of step i-2 has read buffer b
            flat_d.copy_(qkv_h, non_blocking=True)
            in_done[b].record(s_in)
        stream.wait_event(in_done[b])
        oo, ll = fused_attn.forward(qd, kd, vd, is_causal=cfg.causal, scale=scale, return_lse=True)
        buf_free[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(buf_free[b])
            oh.copy_(oo, non_blocking=True)
            lh.copy_(ll, non_blocking=True)
        oo.record_stream(s_out)
        ll.record_stream(s_out)

    e2e_steps = max(1, min(args.steps, 200))
    for i in range(max(2, min(args.warmup, 5))):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record(s_out)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    # This box's PCIe ceiling for the same upload: one copy of the step's q, k, v bytes, timed
    # alone (box to box it has measured 47-55 GB/s); the e2e step cannot beat bytes / that rate.
    h2d_bytes = qkv_h.numel() * qkv_h.element_size()
    with torch.cuda.stream(s_in):
        for _ in range(3):
            dbuf[0][0].copy_(qkv_h, non_blocking=True)
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(s_in)
        for _ in range(20):
            dbuf[0][0].copy_(qkv_h, non_blocking=True)
        p1.record(s_in)
    torch.cuda.synchronize()
    pcie_h2d_gbs = h2d_bytes * 20 / (p0.elapsed_time(p1) * 1e-3) / 1e9
    clocks = sampler.stop() if sampler else None

    err, bits = fused_attn.last_device_error()
    if err != 0:
        raise SystemExit(f"device status after timing: {err} bits={bits:#x}")

    kernel_ms_sum = float(sum(times))
    per_rank = torch.tensor([kernel_ms_sum, e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(per_rank, op=dist.ReduceOp.MAX)
    kernel_ms_sum, e2e_ms = float(per_rank[0]), float(per_rank[1])
    ms_per_step = kernel_ms_sum / args.steps
    flops_rank = attention_flops(cfg.B, cfg.H, cfg.N, cfg.D, cfg.causal)
    flops_job = flops_rank * world
    value = flops_job / (ms_per_step * 1e-3) / 1e12
    e2e_value = flops_job / (e2e_ms * 1e-3) / 1e12

    secondary = None
    cpu_base = None
    c4 = c4_strong(world, rank, dev, stream, flush, max(5, min(args.steps, 20)), args.warmup) \
        if not args.quick and base.name != "C4" else None
    if rank == 0 and world == 1 and not args.quick:
        secondary = secondary_measurements(cfg, q, k, v, flush, stream, max(20, min(args.steps, 200)))
        cpu_base = cpu_sample(cfg, args.cpu_budget, threads=_host_threads())
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    peak, peak_src = load_peaks()
    achieved = flops_rank / (ms_per_step * 1e-3) / 1e12  # one launch on one GPU
    dt = {torch.float16: "fp16", torch.bfloat16: "bf16"}[cfg.dtype]
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": dt,
        "data": f"synthetic: torch.randn iid N(0,1), seed {cfg.seed}(+rank), [B,H,N,D] contiguous",
        "config": config,
        "roofline": {
            "bound": "tensor",
            "achieved": achieved,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": achieved / peak,
            "traffic": profile_traffic(base.name if base.name != "C3" else "C3"),
            "peak_source": peak_src,
            "algorithmic_bytes": attention_bytes(cfg.B, cfg.H, cfg.hkv, cfg.N, cfg.D, 2),
            "algorithmic_flops": flops_rank,
        },
        "cpu_baseline": cpu_base,
        "e2e": {
            "value": e2e_value,
            "unit": UNIT,
            "h2d_bytes_per_step": int(qkv_h.numel() * qkv_h.element_size()),
            "d2h_bytes_per_step": int(o.numel() * o.element_size() + lse.numel() * lse.element_size()),
            "ms_per_step": e2e_ms,
            "steps": e2e_steps,
            "h2d_gbs": h2d_bytes / (e2e_ms * 1e-3) / 1e9,
            "pcie_h2d_gbs_one_copy": pcie_h2d_gbs,
            "api": "fused_attn.forward (torch.ops.fused_attn.forward) from pinned host memory: "
                   "q, k, v uploaded in one copy from one pinned buffer, O and LSE downloaded; "
                   "double-buffered: upload / kernel / download on three streams",
        },
        "gpu_launches": args.steps,
        "clocks": clocks,
        "kernel_ms": {"median": statistics.median(times), "p10": _pct(times, 10),
                      "p90": _pct(times, 90), "min": min(times)},
        "secondary": dict(secondary or {}, **({"c4_strong": c4} if c4 else {})) or None,
    }
    print(json.dumps(line), flush=True)
    return 0


def c4_strong(world: int, rank: int, dev, stream, flush, steps: int, warmup: int) -> dict:
    """secondary.c4_strong: C4 (B1 H32 N16384 D128 bf16 causal, seed 3) split by heads over the
    ranks (fused_attn.sharding: 32/world contiguous heads each, no collective on the data path),
    max-over-ranks device time; then O and LSE of every rank are all-gathered (off the hot path)
    and rank 0 compares them with one launch over all 32 heads on its own GPU, which it also
    times (strong-scaling efficiency = one-GPU time / (world x sharded time))."""
    import torch
    import torch.distributed as dist

    from fused_attn import sharding

    wl = workloads()
    base = wl.CONFIGS["C4"]
    if base.H % world:
        return {"skipped": f"{base.H} heads do not split evenly over {world} ranks"}
    q_all, k_all, v_all = wl.make_qkv(base.B, base.H, base.N, base.D, dtype=base.dtype,
                                      seed=base.seed)
    h0, h1 = sharding.head_range(base.H, world, rank)
    q, k, v = (t.to(dev) for t in sharding.shard_heads(q_all, k_all, v_all, world, rank))
    scale = 1.0 / math.sqrt(base.D)
    op = torch.ops.fused_attn.forward
    if world > 1:
        dist.barrier()
    times = time_kernel(lambda: op(q, k, v, True, scale), steps, max(3, min(warmup, 5)), flush,
                        stream)
    t = torch.tensor([sum(times)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0]) / steps
    o, lse = op(q, k, v, True, scale)
    torch.cuda.synchronize()
    if world > 1:
        o, lse = sharding.gather_heads(o, world), sharding.gather_heads(lse, world)
    flops = wl.attention_flops(base.B, base.H, base.N, base.D, True)
    out = {"workload": base.label(), "heads_per_gpu": h1 - h0, "ranks": world,
           "ms_max_over_ranks": ms, "tflops": flops / ms / 1e9,
           "protocol": f"{steps} launches per rank, CUDA events on the launching stream, L2 "
                       "flushed before each (inputs > L2 anyway); max over ranks"}
    if rank == 0:
        qf, kf, vf = (t.to(dev) for t in (q_all, k_all, v_all))
        t1 = time_kernel(lambda: op(qf, kf, vf, True, scale), steps, 3, flush, stream)
        of, lf = op(qf, kf, vf, True, scale)
        torch.cuda.synchronize()
        ms1 = sum(t1) / steps
        out.update({"one_gpu_ms": ms1, "one_gpu_tflops": flops / ms1 / 1e9,
                    "efficiency_vs_one_gpu": ms1 / (world * ms),
                    "o_bitwise_equal_to_one_launch": bool(torch.equal(o, of)),
                    "lse_bitwise_equal_to_one_launch": bool(torch.equal(lse, lf))})
        del qf, kf, vf, of, lf
    del q, k, v, o, lse
    torch.cuda.empty_cache()
    return out


def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def _pct(xs, p):
    s = sorted(xs)
    return s[min(len(s) - 1, max(0, int(round(p / 100 * (len(s) - 1)))))]


def secondary_measurements(cfg, q, k, v, flush, stream, steps):
    """Context numbers (not the headline): PyTorch SDPA on the same inputs and the same
    protocol, a CUDA-graph batch average of our kernel, the D64 (C2) configs, the fp32 (stage 3)
    configs and the GPT-2 block (C5)."""
    import torch
    import torch.nn.functional as F

    wl = workloads()
    CONFIGS, attention_flops, make_qkv = wl.CONFIGS, wl.attention_flops, wl.make_qkv

    out = {}
    fl = attention_flops(cfg.B, cfg.H, cfg.N, cfg.D, cfg.causal)
    scale = 1.0 / math.sqrt(cfg.D)
    t = time_kernel(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=cfg.causal),
                    steps, 10, flush, stream)
    ms = statistics.median(t)
    out["torch_sdpa_same_gpu"] = {"ms_median": ms, "tflops": fl / ms / 1e9,
                                  "note": "F.scaled_dot_product_attention default backend"}
    t = time_kernel(lambda: torch.ops.fused_attn.forward(q, k, v, cfg.causal, scale), steps, 10,
                    flush, stream)
    ms = statistics.median(t)
    out["ours_median"] = {"ms_median": ms, "tflops": fl / ms / 1e9}
    # Every SDPA backend that accepts each BASELINE shape, same protocol (the reference's bench
    # times EFFICIENT, FLASH, cuDNN: bench/bench.py:279-356); ours against the best of them.
    for name in ("C3", "C3bf16", "C2", "C2c"):
        c = CONFIGS[name]
        if name == cfg.name:
            q2, k2, v2 = q, k, v
        else:
            q2, k2, v2 = make_qkv(c.B, c.H, c.N, c.D, dtype=c.dtype, seed=c.seed, device=q.device)
        out[f"sdpa_backends_{name}"] = sdpa_backends(c, q2, k2, v2, flush, stream, steps)
    # The C3 N sweep of the baseline (same B, H, D, seed), fp16 and bf16.
    sweep = {}
    for n in wl.C3_SWEEP_N:
        for dt in (torch.float16, torch.bfloat16):
            c = wl.Config("C3", 2, 8, n, 128, dt, 2, True)
            q2, k2, v2 = make_qkv(c.B, c.H, c.N, c.D, dtype=c.dtype, seed=c.seed, device=q.device)
            r = sdpa_backends(c, q2, k2, v2, flush, stream, min(steps, 50))
            sweep[c.label()] = {k: r[k] for k in ("ours_tflops", "best_sdpa", "best_sdpa_tflops",
                                                  "ours_over_best_sdpa") if k in r}
            del q2, k2, v2
    out["c3_sweep"] = sweep
    # CUDA-graph batch of 20 launches (no flush in between: warm L2), labelled as such.
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        torch.ops.fused_attn.forward(q, k, v, cfg.causal, scale)
        with torch.cuda.graph(g, stream=s):
            for _ in range(20):
                torch.ops.fused_attn.forward(q, k, v, cfg.causal, scale)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 100
    out["ours_cuda_graph_batch20_warm_l2"] = {"ms": ms, "tflops": fl / ms / 1e9}
    del g
    for name in ("C2", "C2c"):
        c = CONFIGS[name]
        q2, k2, v2 = make_qkv(c.B, c.H, c.N, c.D, dtype=c.dtype, seed=c.seed, device=q.device)
        f2 = attention_flops(c.B, c.H, c.N, c.D, c.causal)
        s2 = 1.0 / math.sqrt(c.D)
        t = time_kernel(lambda: torch.ops.fused_attn.forward(q2, k2, v2, c.causal, s2), steps, 10,
                        flush, stream)
        ts = time_kernel(lambda: F.scaled_dot_product_attention(q2, k2, v2, is_causal=c.causal),
                         steps, 10, flush, stream)
        out[name] = {"workload": c.label(), "ours_ms": statistics.median(t),
                     "ours_tflops": f2 / statistics.median(t) / 1e9,
                     "sdpa_ms": statistics.median(ts), "sdpa_tflops": f2 / statistics.median(ts) / 1e9}
    # fp32 inputs (stage 3: tf32 tensor cores after the tf32-rounding pre-pass into the
    # workspace): the C1 configuration and the C3 shape in fp32.
    for name, (b_, h_, n_, d_, causal_, seed_) in (("C1c_fp32", (1, 2, 128, 64, True, 0)),
                                                   ("C3_shape_fp32", (2, 8, 2048, 128, True, 2))):
        q3, k3, v3 = make_qkv(b_, h_, n_, d_, dtype=torch.float32, seed=seed_, device=q.device)
        f3 = attention_flops(b_, h_, n_, d_, causal_)
        s3 = 1.0 / math.sqrt(d_)
        t = time_kernel(lambda: torch.ops.fused_attn.forward(q3, k3, v3, causal_, s3), steps, 10,
                        flush, stream)
        ts = time_kernel(lambda: F.scaled_dot_product_attention(q3, k3, v3, is_causal=causal_),
                         steps, 10, flush, stream)
        out[name] = {"workload": f"B{b_}H{h_}N{n_}D{d_} fp32 {'causal' if causal_ else 'full'}",
                     "path": "stage 3: tf32 rounding pre-pass + tcgen05 kind::tf32",
                     "ours_ms": statistics.median(t), "ours_tflops": f3 / statistics.median(t) / 1e9,
                     "sdpa_fp32_ms": statistics.median(ts),
                     "sdpa_fp32_tflops": f3 / statistics.median(ts) / 1e9}
    out["C5_gpt2_block"] = gpt_block_measurements(q.device)
    return out


def sdpa_backends(c, q, k, v, flush, stream, steps) -> dict:
    """TFLOP/s of our op and of each PyTorch SDPA backend (FLASH, cuDNN, EFFICIENT) that accepts
    the shape, on the same inputs and protocol; `best_sdpa` and our ratio to it."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    fl = workloads().attention_flops(c.B, c.H, c.N, c.D, c.causal)
    scale = 1.0 / math.sqrt(c.D)
    res = {"workload": c.label()}
    t = time_kernel(lambda: torch.ops.fused_attn.forward(q, k, v, c.causal, scale), steps, 10,
                    flush, stream)
    res["ours_tflops"] = fl / statistics.median(t) / 1e9
    best = None
    for name, be in (("flash", SDPBackend.FLASH_ATTENTION), ("cudnn", SDPBackend.CUDNN_ATTENTION),
                     ("efficient", SDPBackend.EFFICIENT_ATTENTION)):
        try:
            with sdpa_kernel([be]):
                F.scaled_dot_product_attention(q, k, v, is_causal=c.causal)
                t = time_kernel(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=c.causal),
                                steps, 10, flush, stream)
        except RuntimeError as e:
            res[f"sdpa_{name}"] = {"refused": str(e).splitlines()[0][:120]}
            continue
        tf = fl / statistics.median(t) / 1e9
        res[f"sdpa_{name}_tflops"] = tf
        if best is None or tf > best[1]:
            best = (name, tf)
    if best is not None:
        res["best_sdpa"] = best[0]
        res["best_sdpa_tflops"] = best[1]
        res["ours_over_best_sdpa"] = res["ours_tflops"] / best[1]
    return res


def gpt_block_measurements(device, warmup: int = 10, iters: int = 50) -> dict:
    """C5: tokens/s of the GPT-2-small block (token + position embedding, one pre-LN block,
    d 768, 12 heads of 64, MLP 4x, fp16, batch 16 x T 1024) with the attention through our op
    (strided views, and the reference's .contiguous() binding path) and through PyTorch SDPA,
    plus the attention window's share.  Warm, no L2 flush -- the reference harness's protocol
    for this end-to-end row (bench/gpt_block.py), whose own block takes a random x at batch 8."""
    import torch

    from fused_attn import gpt_block as gb

    cfg = gb.GPTConfig()
    ids = gb.token_ids(cfg, device)
    impls = {}
    for impl in ("fused_strided", "fused_contiguous", "sdpa_flash", "sdpa_cudnn"):
        try:
            model = gb.build_model(cfg, impl, device)
            m = gb.measure(model, ids, warmup, iters)
        except RuntimeError as e:  # an SDPA backend that refuses the shape
            impls[impl] = {"refused": str(e).splitlines()[0][:160]}
            continue
        impls[impl] = {k: round(v, 4) for k, v in m.items()}
        del model
        torch.cuda.empty_cache()
    return {"workload": f"GPT-2-small block B{cfg.batch} T{cfg.seq} d{cfg.n_embd} "
                        f"H{cfg.n_head} D{cfg.head_dim} fp16 causal, token+position embedding",
            "metric": "tokens/s", "protocol": f"warm, no L2 flush, {warmup} warm-up + {iters} "
                                              "timed forwards, CUDA-event median",
            "attention_gflop": cfg.attention_flops() / 1e9, "gemm_gflop": cfg.gemm_flops() / 1e9,
            "impls": impls}


def _cmd_version(cmd: list[str], pick) -> str:
    try:
        out = subprocess.run(cmd, capture_output=True, text=True, timeout=20).stdout
        return pick(out)
    except (OSError, subprocess.SubprocessError, IndexError, ValueError):
        return "unknown"


def run_sweep(args) -> int:
    """--sweep OUT.csv: the reference's canonical sweep (CONTRACT.md §5: N in 128..4096, D in
    {64, 128}, (B, H) in {(1, 8), (8, 32)}, causal 0/1; fp16) plus C3 in bf16, for our kernel and
    every PyTorch SDPA backend that accepts the shape, written as rows of the reference's frozen
    CSV schema (fused_attn/benchcsv.py) and rendered to OUT.md.  Our rows carry max_abs against
    fp32 SDPA on the same inputs."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from fused_attn import benchcsv
    from fused_attn.workloads import make_qkv

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 << 18, dtype=torch.float32, device=dev)
    env = {
        "commit": args.commit,
        "gpu": torch.cuda.get_device_name(0),
        "driver": _cmd_version(["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader",
                                "--id=0"], lambda o: o.strip().splitlines()[0]),
        "nvcc": _cmd_version(["nvcc", "--version"],
                             lambda o: o.split("release")[1].split(",")[0].strip()),
        "torch": torch.__version__,
        "ncu": _cmd_version(["ncu", "--version"], lambda o: o.strip().splitlines()[-1].split()[-1]),
        "clock_mhz": "unlocked",
    }
    backends = {"sdpa_flash": SDPBackend.FLASH_ATTENTION,
                "sdpa_efficient": SDPBackend.EFFICIENT_ATTENTION,
                "sdpa_cudnn": SDPBackend.CUDNN_ATTENTION}
    shapes = [(b, h, n, d, c, torch.float16) for (b, h) in ((1, 8), (8, 32))
              for n in (128, 256, 512, 1024, 2048, 4096) for d in (64, 128) for c in (False, True)]
    shapes.append((2, 8, 2048, 128, True, torch.bfloat16))
    rows = []
    clocks = ClockSampler(0)
    clocks.start()
    t_start = time.time()
    for (b, h, n, d, causal, dt) in shapes:
        dname = {torch.float16: "fp16", torch.bfloat16: "bf16"}[dt]
        q, k, v = make_qkv(b, h, n, d, dtype=dt, device=dev, seed=2)
        scale = 1.0 / math.sqrt(d)
        with sdpa_kernel([SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]):
            ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)
        o = torch.ops.fused_attn.forward(q, k, v, causal, scale)[0]
        err = float((o.float() - ref).abs().max())

        def timed(fn):
            # A short idle before each series lets the clocks recover from the previous (power-
            # capped) one, so rows do not inherit their predecessor's clock state; the SM clock
            # sampled over the series goes into the row's notes.
            torch.cuda.synchronize()
            time.sleep(args.sweep_settle)
            t0 = time.time()
            t = time_kernel(fn, args.sweep_iters, 10, flush, stream)
            mhz = clocks.median_between(t0, time.time())
            return t, ([f"clock_mhz={mhz:.0f}"] if mhz else [])

        t, cn = timed(lambda: torch.ops.fused_attn.forward(q, k, v, causal, scale))
        rows.append(benchcsv.make_row(env, "tuned", dname, b, h, n, d, causal, t,
                                      [f"max_abs={err:.3e}", "vs=sdpa_fp32"] + cn))
        for name, be in backends.items():
            try:
                with sdpa_kernel([be]):
                    F.scaled_dot_product_attention(q, k, v, is_causal=causal)
                    t, cn = timed(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=causal))
            except RuntimeError:
                continue  # the backend refuses this shape/dtype: no row
            rows.append(benchcsv.make_row(env, name, dname, b, h, n, d, causal, t, cn))
        del q, k, v, ref, o
    clocks.window(t_start, time.time())
    clocks.stop()
    benchcsv.write_rows(args.sweep, rows)
    md = Path(args.sweep).with_suffix(".md")
    md.write_text(benchcsv.to_markdown(rows))
    hdr, back = benchcsv.read_rows(args.sweep)
    problems = benchcsv.validate(hdr, back, roof_tflops=_roof_tflops())
    print(json.dumps({"sweep": str(args.sweep), "rows": len(rows), "problems": problems[:10]}))
    return 0 if not problems else 1


def _roof_tflops() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["bf16_tflops"])
    except (OSError, ValueError, KeyError):
        return 1590.0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="C3", help="C3 (default), C3bf16, C2, C2c or C4")
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of CPU oracle work for the cpu_baseline sample")
    ap.add_argument("--quick", action="store_true", help="skip secondary and CPU measurements")
    ap.add_argument("--sweep", default=None,
                    help="write the reference-schema sweep CSV (and .md) to this path instead")
    ap.add_argument("--sweep-iters", type=int, default=100)
    ap.add_argument("--sweep-settle", type=float, default=0.3,
                    help="idle seconds before each timed series of the sweep")
    ap.add_argument("--commit", default="unknown", help="commit SHA recorded in sweep rows")
    args = ap.parse_args(argv)
    if args.sweep:
        return run_sweep(args)
    args.warmup = max(args.warmup, 3)  # the timing rules require at least 3 warm-up steps
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
