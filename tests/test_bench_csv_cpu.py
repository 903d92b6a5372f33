"""Benchmark CSV tooling (fused_attn/benchcsv.py) -- the reference's frozen schema
(CONTRACT.md §3), its row sanity checks (tests/test_bench_sanity.py) and the table generator
(scripts/bench_to_md.py), on CPU.

* the checks accept a well-formed row and catch each kind of bad row;
* the committed sweep (profiles/bench_sweep_b200.csv, produced on a B200 by
  ``python bench.py --sweep``) passes every check, and the committed table next to it is exactly
  what the generator renders from it (a stale table fails, like the reference's docs test).
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest

from fused_attn import benchcsv

ROOT = Path(__file__).resolve().parent.parent
SWEEP = ROOT / "profiles" / "bench_sweep_b200.csv"
ENV = {"commit": "0123abc", "gpu": "NVIDIA B200", "driver": "580.159", "nvcc": "12.9",
       "torch": "2.11.0", "ncu": "2025.2", "clock_mhz": "unlocked"}


def _good_rows():
    t = [0.0300 + 0.0001 * (i % 5) for i in range(100)]
    ours = benchcsv.make_row(ENV, "tuned", "fp16", 2, 8, 2048, 128, True, t,
                             ["max_abs=9.5e-04", "vs=sdpa_fp32"])
    sdpa = benchcsv.make_row(ENV, "sdpa_flash", "fp16", 2, 8, 2048, 128, True,
                             [x * 1.1 for x in t], [])
    return [ours, sdpa]


def test_schema_is_the_references():
    assert benchcsv.SCHEMA == ["commit", "gpu", "driver", "nvcc", "torch", "ncu", "clock_mhz",
                               "impl", "stage", "dtype", "B", "H", "N", "D", "causal",
                               "ms_median", "ms_p10", "ms_p90", "tflops", "gbps", "notes"]


def test_good_rows_pass_and_roundtrip(tmp_path):
    rows = _good_rows()
    p = tmp_path / "s.csv"
    benchcsv.write_rows(p, rows)
    header, back = benchcsv.read_rows(p)
    assert benchcsv.validate(header, back, roof_tflops=1656.4) == []
    assert float(back[0]["tflops"]) == pytest.approx(17.179869184e9 / 0.0302e-3 / 1e12, rel=0.01)
    assert "flops=causal_half" in back[0]["notes"] and back[0]["stage"] == "5"
    md = benchcsv.to_markdown(back)
    assert "| B2 H8 N2048 D128 | 1 |" in md and "sdpa_flash" in md and "1.10x" in md


@pytest.mark.parametrize("mutate,needle", [
    (lambda r: r.update(tflops="999.000"), "does not recompute"),
    (lambda r: r.update(commit="0123abc-dirty"), "clean SHA"),
    (lambda r: r.update(notes="iters=100;flops=causal_half"), "correctness note"),
    (lambda r: r.update(notes=r["notes"].replace("iters=100", "iters=20")), "timed iterations"),
    (lambda r: r.update(ms_p90="0.0900"), "noisy"),
    (lambda r: r.update(impl="stage9"), "unknown impl"),
    (lambda r: r.update(stage="3"), "does not match impl"),
])
def test_bad_rows_are_caught(mutate, needle):
    rows = _good_rows()
    mutate(rows[0])
    problems = benchcsv.validate(list(benchcsv.SCHEMA), rows, roof_tflops=1656.4)
    assert any(needle in p for p in problems), problems


def test_rows_above_the_roof_are_caught():
    rows = _good_rows()
    assert benchcsv.validate(list(benchcsv.SCHEMA), rows, roof_tflops=100.0)


@pytest.mark.skipif(not SWEEP.exists(), reason="no sweep committed yet")
def test_committed_sweep_is_sane_and_its_table_is_current():
    header, rows = benchcsv.read_rows(SWEEP)
    peaks = ROOT / "MEASURED_PEAKS.json"
    roof = json.loads(peaks.read_text())["bf16_tflops"] if peaks.exists() else 1590.0
    assert benchcsv.validate(header, rows, roof_tflops=roof) == []
    assert {r["impl"] for r in rows} >= {"tuned"}
    assert SWEEP.with_suffix(".md").read_text() == benchcsv.to_markdown(rows)


def test_clock_record_falls_back_to_fast_nvml_samples():
    """A timed region shorter than nvidia-smi's 50 ms period gets no nvidia-smi sample; the clock
    record then comes from the ~2 ms NVML samples inside the region (median SM clock, union of
    the throttle reasons seen)."""
    import bench

    c = bench.ClockSampler(0)
    # stop() only needs a process handle that can be terminated
    c.proc = type("P", (), {"terminate": lambda self: None, "wait": lambda self, timeout=None: 0})()
    c.samples = [(0.0, ["0", "1965", "1965", "300", "0x0", "Not Active", "Not Active",
                        "Not Active", "Not Active"])]
    c.fast = [(10.001, 1965.0, 1965.0, 0x0), (10.003, 1950.0, 1965.0, 0x4),
              (10.005, 1965.0, 1965.0, 0x0), (11.0, 900.0, 1965.0, 0x8)]
    c.window(10.0, 10.01)
    rec = c.stop()
    assert rec["samples_in_timed_region"] == 3
    assert rec["sm_mhz"] == 1965.0 and rec["sm_max_mhz"] == 1965.0
    assert rec["reasons"] == ["sw_power_cap"]
    assert "NVML" in rec["source"]
