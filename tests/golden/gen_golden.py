"""Generate the golden fixtures in this directory from the REFERENCE's own implementations.

Run (in a container where the reference tree is present, after ``make -C oracle ref``)::

    python tests/golden/gen_golden.py [--reference-root DIR]   (default: $FA_REFERENCE_ROOT, else
                                                               a `reference` dir beside the repo)

Two independent reference implementations produce every expected output:

* ``oracle/_ref/libfa_ref.so`` -- the reference's src/reference/cpu_reference.cpp compiled
  where it lies (fa::ref::attention_rows, fp64);
* ``python/fused_attn/reference.py::math_reference`` of the reference, imported by file path
  (it needs only torch), fp64.

Inputs come from the reference's seeded generator (tests/conftest.py:99-127: CPU torch.randn in
q, k, v order), stored in the dtype the kernel consumes.  The fixtures are read by
tests/test_oracle_cpu.py (to pin the C restatement in oracle/fa_oracle.c) and by
tests/test_kernels_gpu.py (to check the sm_100a kernel against values the reference produced).
Nothing at test time reads the reference tree.
"""

from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "fused-attention-cuda_b200"))

import oracle  # noqa: E402
from fused_attn.workloads import make_qkv  # noqa: E402

# name, (B, H, Hkv, N, D), dtype, seed, scale (None = 1/sqrt(D))
CASES = [
    ("c1_fp32", (1, 2, 2, 128, 64), torch.float32, 0, None),
    ("fp16_n64", (1, 2, 2, 64, 64), torch.float16, 1, None),
    ("bf16_n96_d128", (1, 1, 1, 96, 128), torch.bfloat16, 5, None),
    ("gqa_fp32", (1, 4, 2, 64, 64), torch.float32, 17, None),
    ("fp16_scale005_d128", (1, 1, 1, 64, 128), torch.float16, 15, 0.05),
]


def load_reference_py(root: Path):
    path = root / "python" / "fused_attn" / "reference.py"
    spec = importlib.util.spec_from_file_location("ref_fused_attn_reference", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default=str(oracle.reference_root()))
    ap.add_argument("--out", default=str(HERE / "golden.npz"))
    args = ap.parse_args()
    if not (Path(args.reference_root) / "python" / "fused_attn" / "reference.py").exists():
        ap.error(f"no reference checkout at {args.reference_root}: pass --reference-root or set "
                 "FA_REFERENCE_ROOT")
    ref_py = load_reference_py(Path(args.reference_root))
    if not oracle.ref_available():
        oracle.build(ref=True)
    arrays: dict[str, np.ndarray] = {}
    for name, (b, h, hkv, n, d), dtype, seed, scale in CASES:
        q, k, v = make_qkv(b, h, n, d, dtype=dtype, hkv=hkv, seed=seed)
        store = {torch.float32: np.float32, torch.float16: np.float16}.get(dtype)
        for t, tn in ((q, "q"), (k, "k"), (v, "v")):
            if store is not None:
                arrays[f"{name}/{tn}"] = t.numpy().astype(store)
            else:  # bf16: numpy has no bf16; store the exact values as fp32
                arrays[f"{name}/{tn}"] = t.float().numpy()
        arrays[f"{name}/meta"] = np.array(
            [b, h, hkv, n, d, seed, {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype]],
            dtype=np.int64)
        arrays[f"{name}/scale"] = np.array([np.nan if scale is None else scale], dtype=np.float64)
        for causal in (False, True):
            tag = "causal" if causal else "full"
            o_c, lse_c, _ = oracle.ref_attention(q, k, v, causal=causal, scale=scale, threads=4)
            o_py, lse_py = ref_py.math_reference(q, k, v, is_causal=causal, scale=scale)
            d_o = float(np.abs(o_c - o_py.numpy()).max())
            d_l = float(np.abs(lse_c - lse_py.numpy()).max())
            if not (d_o < 1e-10 and d_l < 1e-10):
                raise SystemExit(f"{name}/{tag}: the two reference oracles disagree ({d_o}, {d_l})")
            arrays[f"{name}/{tag}/o"] = o_c
            arrays[f"{name}/{tag}/lse"] = lse_c
            print(f"{name}/{tag}: cpu_reference vs reference.py max|do|={d_o:.2e} max|dlse|={d_l:.2e}")
    np.savez_compressed(args.out, **arrays)
    print(f"wrote {args.out} ({Path(args.out).stat().st_size / 1024:.0f} KiB)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
