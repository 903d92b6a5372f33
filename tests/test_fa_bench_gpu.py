"""The torch-free C++ harness (fused_attn/fa_bench, csrc/fa_bench.cpp) on the GPU.

Reference counterpart: the reference's fa_bench (bench/bench_main.cu), which writes a timing row
only after its fp64 self-check passed (:589-656, :763).  These tests run the harness as a separate
process -- it links libfa_sm100.so through include/fa_sm100.h alone -- and check that:

* at C3 (B2 H8 N2048 D128 fp16 causal) its self-check passes and its median kernel time is within
  10 % of the same launch timed through the PyTorch op with bench.py's protocol;
* bf16 passes the check too;
* a planted disagreement (a constant added to the oracle's output on the CPU) makes it refuse the
  row: exit status 2 and nothing on stdout.
"""

from __future__ import annotations

import json
import math
import statistics
import subprocess

import pytest
import torch

import fused_attn
from conftest import ROOT
from fused_attn.workloads import make_qkv

pytestmark = pytest.mark.gpu

HARNESS = ROOT / "fused-attention-cuda_b200" / "fused_attn" / "fa_bench"


def run(*args, timeout=600):
    if not HARNESS.exists():
        pytest.skip("fa_bench is not built (python fused-attention-cuda_b200/build.py)")
    return subprocess.run([str(HARNESS), *args], capture_output=True, text=True, timeout=timeout)


def test_c3_row_passes_self_check_and_matches_bench_timing():
    r = run("--cfg", "B2_H8_N2048_D128", "--dtype", "fp16", "--causal", "1", "--iters", "200",
            "--warmup", "10")
    assert r.returncode == 0, r.stderr
    row = json.loads(r.stdout.strip().splitlines()[-1])
    assert row["self_check"]["passed"] is True
    assert row["self_check"]["max_abs_o"] <= 2e-3 and row["self_check"]["max_abs_lse"] <= 1e-3
    # The same launch through the PyTorch op, bench.py's timing protocol (256 MiB flush, one event
    # pair per launch on the launching stream, median).
    import bench

    q, k, v = make_qkv(2, 8, 2048, 128, dtype=torch.float16, device="cuda", seed=2)
    flush = torch.empty(bench.FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    scale = 1.0 / math.sqrt(128)
    t = bench.time_kernel(lambda: torch.ops.fused_attn.forward(q, k, v, True, scale), 200, 10,
                          flush, stream)
    ours = statistics.median(t)
    assert abs(row["median_ms"] - ours) <= 0.10 * ours, (row["median_ms"], ours)


def test_bf16_row_passes_self_check():
    r = run("--cfg", "B1_H4_N1024_D64", "--dtype", "bf16", "--causal", "0", "--iters", "20")
    assert r.returncode == 0, r.stderr
    row = json.loads(r.stdout.strip().splitlines()[-1])
    assert row["self_check"]["passed"] is True and row["self_check"]["max_abs_o"] <= 8e-3


def test_row_refused_when_the_check_fails():
    r = run("--cfg", "B1_H2_N256_D128", "--dtype", "fp16", "--iters", "5",
            "--perturb-oracle", "0.05")
    assert r.returncode == 2
    assert r.stdout.strip() == ""
    assert "row refused" in r.stderr
    assert fused_attn.is_available()
