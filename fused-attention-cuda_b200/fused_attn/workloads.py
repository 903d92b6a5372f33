"""Seeded synthetic workloads and the FLOP / byte models of the SDPA forward.

* ``make_qkv`` is the reference's input generator (tests/conftest.py:99-127): ``torch.randn``
  on the CPU from ``torch.Generator().manual_seed(seed)`` in q, k, v order, scaled, then cast
  and moved.  The same (seed, shape) gives the same values on every machine; only the final
  rounding to the kernel dtype differs.
* ``CONFIGS`` are the configurations the benchmark and the parity tests run (C1..C5), with the
  shapes, dtypes and seeds named by the benchmark baseline.  No public dataset is involved: the
  inputs are iid N(0, 1), as the reference generates them.
* ``attention_flops`` follows scripts/fa_common.py:250-256: 4*B*H*N^2*D, halved for causal.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


def make_qkv(b: int, h: int, n: int, d: int, dtype: torch.dtype = torch.float32,
             device: str | torch.device = "cpu", hkv: int | None = None, seed: int = 0,
             scale_inputs: float = 1.0):
    gen = torch.Generator(device="cpu").manual_seed(seed)
    hkv = h if hkv is None else hkv
    q = torch.randn(b, h, n, d, generator=gen, dtype=torch.float32)
    k = torch.randn(b, hkv, n, d, generator=gen, dtype=torch.float32)
    v = torch.randn(b, hkv, n, d, generator=gen, dtype=torch.float32)
    return tuple((t * scale_inputs).to(device=device, dtype=dtype).contiguous() for t in (q, k, v))


def attention_flops(b: int, h: int, n: int, d: int, causal: bool) -> float:
    f = 4.0 * b * h * n * n * d
    return f / 2.0 if causal else f


def attention_bytes(b: int, h: int, hkv: int, n: int, d: int, elem_bytes: int) -> float:
    """Algorithmic HBM bytes: read Q, K, V once, write O and LSE once
    (bench/bench_main.cu:570-581)."""
    return float(elem_bytes) * n * d * (2 * b * h + 2 * b * hkv) + 4.0 * b * h * n


@dataclass(frozen=True)
class Config:
    name: str
    B: int
    H: int
    N: int
    D: int
    dtype: torch.dtype
    seed: int
    causal: bool
    Hkv: int | None = None

    @property
    def hkv(self) -> int:
        return self.H if self.Hkv is None else self.Hkv

    @property
    def flops(self) -> float:
        return attention_flops(self.B, self.H, self.N, self.D, self.causal)

    def label(self) -> str:
        dt = {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32"}[self.dtype]
        c = "causal" if self.causal else "full"
        return f"{self.name} B{self.B}H{self.H}N{self.N}D{self.D} {dt} {c}"


CONFIGS = {
    "C1": Config("C1", 1, 2, 128, 64, torch.float32, 0, False),
    "C1c": Config("C1c", 1, 2, 128, 64, torch.float32, 0, True),
    "C2": Config("C2", 2, 8, 2048, 64, torch.float16, 1, False),
    "C2c": Config("C2c", 2, 8, 2048, 64, torch.float16, 1, True),
    "C3": Config("C3", 2, 8, 2048, 128, torch.float16, 2, True),
    "C3bf16": Config("C3bf16", 2, 8, 2048, 128, torch.bfloat16, 2, True),
    "C4": Config("C4", 1, 32, 16384, 128, torch.bfloat16, 3, True),
}

# The N sweep of C3 (same B/H/D/seed).
C3_SWEEP_N = (512, 1024, 4096, 8192)
