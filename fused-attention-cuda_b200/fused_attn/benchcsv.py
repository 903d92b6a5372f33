"""Benchmark CSV rows in the reference's frozen schema, their sanity checks, and the markdown
table rendered from them.

Reference counterparts: CONTRACT.md §3 (the schema below, column for column), the row checks of
tests/test_bench_sanity.py and the README table of scripts/bench_to_md.py.  The schema is kept
alike so that results from this build drop into the reference's tooling unchanged; the checks
and the renderer are this build's own.

FLOP convention (CONTRACT.md §3): 4·B·H·N²·D, halved for causal rows of tile-skipping kernels
(every implementation benchmarked here skips masked tiles), ``notes`` carries
``flops=causal_half``.  ``gbps`` = modelled minimum bytes / time: Q + K + V + O (+ LSE for our
kernel).
"""

from __future__ import annotations

import csv
import math
from collections import defaultdict
from pathlib import Path

SCHEMA = ("commit,gpu,driver,nvcc,torch,ncu,clock_mhz,impl,stage,dtype,B,H,N,D,causal,"
          "ms_median,ms_p10,ms_p90,tflops,gbps,notes").split(",")
OUR_IMPLS = {"tuned": 5, "fused": 3}
BASELINE_IMPLS = ("sdpa_efficient", "sdpa_flash", "sdpa_math_fp32", "sdpa_cudnn", "torch_unfused",
                  "flash_attn")
DTYPES = ("fp32", "fp16", "bf16")
ELEM_BYTES = {"fp32": 4, "fp16": 2, "bf16": 2}
MIN_ITERS = 100
NOISE_RATIO = 1.25  # p90/p10 above this must be flagged `noisy`
TFLOPS_TOL = 0.01


def flops(B: int, H: int, N: int, D: int, causal: bool) -> float:
    f = 4.0 * B * H * N * N * D
    return f / 2 if causal else f


def min_bytes(B: int, H: int, N: int, D: int, dtype: str, with_lse: bool) -> float:
    b = 4.0 * B * H * N * D * ELEM_BYTES[dtype]
    return b + (4.0 * B * H * N if with_lse else 0.0)


def make_row(env: dict, impl: str, dtype: str, B: int, H: int, N: int, D: int, causal: bool,
             times_ms: list[float], notes: list[str]) -> dict:
    """One row from per-iteration times (ms).  `env` holds commit, gpu, driver, nvcc, torch, ncu,
    clock_mhz."""
    ts = sorted(times_ms)

    def pct(p):
        return ts[min(len(ts) - 1, max(0, int(round(p / 100 * (len(ts) - 1)))))]

    med = pct(50)
    p10, p90 = pct(10), pct(90)
    stage = OUR_IMPLS.get(impl, 0)
    tfl = flops(B, H, N, D, causal) / (med * 1e-3) / 1e12
    gbs = min_bytes(B, H, N, D, dtype, impl in OUR_IMPLS) / (med * 1e-3) / 1e9
    note = list(notes) + [f"iters={len(ts)}"]
    if causal:
        note.append("flops=causal_half")
    if p10 > 0 and p90 / p10 > NOISE_RATIO:
        note.append("noisy")
    row = {k: env.get(k, "") for k in SCHEMA[:7]}
    row.update({"impl": impl, "stage": str(stage), "dtype": dtype, "B": str(B), "H": str(H),
                "N": str(N), "D": str(D), "causal": "1" if causal else "0",
                "ms_median": f"{med:.4f}", "ms_p10": f"{p10:.4f}", "ms_p90": f"{p90:.4f}",
                "tflops": f"{tfl:.3f}", "gbps": f"{gbs:.1f}", "notes": ";".join(note)})
    return row


def write_rows(path: str | Path, rows: list[dict]) -> None:
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=SCHEMA)
        w.writeheader()
        for r in rows:
            w.writerow(r)


def read_rows(path: str | Path) -> tuple[list[str], list[dict]]:
    with open(path, newline="") as f:
        rd = csv.DictReader(f)
        return list(rd.fieldnames or []), list(rd)


def notes_of(row: dict) -> dict[str, str]:
    out: dict[str, str] = {}
    for tok in (row.get("notes") or "").split(";"):
        k, _, v = tok.partition("=")
        if k.strip():
            out.setdefault(k.strip(), v.strip())
    return out


def validate(header: list[str], rows: list[dict], roof_tflops: float | None = None) -> list[str]:
    """Problems with a CSV (empty list = sane): exact schema; known impl/dtype/causal values;
    clean commit; stage matches impl; p10 <= median <= p90 and a noise flag above NOISE_RATIO;
    tflops recomputes from ms_median and the shape within 1 %; >= MIN_ITERS timed iterations;
    a correctness note (`max_abs=`) on every row of our kernels; tflops below the roof."""
    bad: list[str] = []
    if header != SCHEMA:
        return [f"header {header} != schema {SCHEMA}"]
    for i, r in enumerate(rows):
        where = f"row {i + 2} ({r.get('impl')} {r.get('dtype')} B{r.get('B')} H{r.get('H')} " \
                f"N{r.get('N')} D{r.get('D')} c{r.get('causal')})"
        impl = r["impl"]
        if impl not in OUR_IMPLS and impl not in BASELINE_IMPLS:
            bad.append(f"{where}: unknown impl")
            continue
        if r["dtype"] not in DTYPES or r["causal"] not in ("0", "1"):
            bad.append(f"{where}: bad dtype/causal")
            continue
        if not r["commit"] or r["commit"].endswith("-dirty"):
            bad.append(f"{where}: commit must be a clean SHA")
        if int(r["stage"]) != OUR_IMPLS.get(impl, 0):
            bad.append(f"{where}: stage {r['stage']} does not match impl")
        n = notes_of(r)
        try:
            med, p10, p90 = float(r["ms_median"]), float(r["ms_p10"]), float(r["ms_p90"])
            tfl = float(r["tflops"])
        except ValueError:
            bad.append(f"{where}: non-numeric timing")
            continue
        if not (0 < p10 <= med <= p90):
            bad.append(f"{where}: p10 <= median <= p90 violated")
        if p90 / p10 > NOISE_RATIO and "noisy" not in n:
            bad.append(f"{where}: p90/p10 = {p90 / p10:.2f} without a `noisy` flag")
        B, H, N, D = (int(r[k]) for k in ("B", "H", "N", "D"))
        want = flops(B, H, N, D, r["causal"] == "1") / (med * 1e-3) / 1e12
        if abs(want - tfl) > TFLOPS_TOL * max(want, 1e-9):
            bad.append(f"{where}: tflops {tfl} does not recompute ({want:.3f})")
        if int(n.get("iters", "0") or 0) < MIN_ITERS:
            bad.append(f"{where}: fewer than {MIN_ITERS} timed iterations")
        if impl in OUR_IMPLS and "max_abs" not in n:
            bad.append(f"{where}: our row without a correctness note (max_abs=)")
        if roof_tflops is not None and tfl > roof_tflops * 1.05:
            bad.append(f"{where}: {tfl} TFLOP/s above the roof {roof_tflops}")
    return bad


def to_markdown(rows: list[dict]) -> str:
    """One table per dtype: each shape with our kernel's TFLOP/s, the best PyTorch SDPA backend on
    the same GPU and the ratio."""
    by_shape: dict[tuple, dict[str, dict]] = defaultdict(dict)
    for r in rows:
        key = (r["dtype"], int(r["B"]), int(r["H"]), int(r["N"]), int(r["D"]), r["causal"])
        by_shape[key][r["impl"]] = r
    out: list[str] = []
    env = rows[0] if rows else {}
    if rows:
        out.append(f"GPU: {env.get('gpu')} (driver {env.get('driver')}, nvcc {env.get('nvcc')}, "
                   f"torch {env.get('torch')}), commit {env.get('commit')}. CUDA-event median of "
                   f">= {MIN_ITERS} launches, L2 flushed before each; TFLOP/s = 4*B*H*N^2*D "
                   "(halved for causal).")
        out.append("")
    for dt in DTYPES:
        keys = sorted(k for k in by_shape if k[0] == dt)
        if not keys:
            continue
        out.append(f"| {dt} shape | causal | ours ms | ours TFLOP/s | best SDPA backend | "
                   "SDPA TFLOP/s | ours / SDPA |")
        out.append("|---|---|---|---|---|---|---|")
        for k in keys:
            impls = by_shape[k]
            ours = next((impls[i] for i in OUR_IMPLS if i in impls), None)
            base = [impls[i] for i in BASELINE_IMPLS if i in impls]
            best = max(base, key=lambda r: float(r["tflops"]), default=None)
            _, B, H, N, D, c = k
            o_ms = ours["ms_median"] if ours else "-"
            o_tf = ours["tflops"] if ours else "-"
            b_name = best["impl"] if best else "-"
            b_tf = best["tflops"] if best else "-"
            ratio = (f"{float(ours['tflops']) / float(best['tflops']):.2f}x"
                     if ours and best and float(best["tflops"]) > 0 else "-")
            out.append(f"| B{B} H{H} N{N} D{D} | {c} | {o_ms} | {o_tf} | {b_name} | {b_tf} | "
                       f"{ratio} |")
        out.append("")
    return "\n".join(out).rstrip() + "\n"


def geomean(xs: list[float]) -> float:
    xs = [x for x in xs if x > 0]
    return math.exp(sum(math.log(x) for x in xs) / len(xs)) if xs else float("nan")
