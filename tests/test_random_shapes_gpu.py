"""Seeded random shapes against the fp64 oracle (the parity cases carry the marker ``gpu``).

Each case draws batch, query and kv heads (GQA/MQA ratios 1-4), a sequence length that is a
multiple of 32 but usually not of the 64/128-key tiles, head dim, causal or full, fp16 or bf16, a
non-default softmax scale or input magnitude (peaked rows: large running-max jumps), which kernel
runs (the default choice or a forced key-tile width: the lookahead kernel, the 128-key and the
32-key kernel) and whether q/k/v arrive as contiguous tensors or as strided [B, T, H, D] views.
Every case is gated against the oracle run on the same rounded inputs, LSE within the dtype's
LSE tolerance.  Unit-variance inputs (the distribution the tolerances are stated for): every O
element within the dtype's tolerance or, where larger, half a unit in the last place of the
reference value in the output dtype plus 2e-3 (the stated bf16 extension: rows that average one
to three keys can reach |O| >= 4, where bf16's own rounding is 1.56e-2).  Inputs scaled by 2
(|V| up to ~8, peaked rows): the reference's gate for such data -- the error at most twice that of
PyTorch's own unfused attention in the same dtype plus 1e-6 (the ratio rule), and at most the
dtype's cap relative to max|O|.
"""

from __future__ import annotations

import random

import numpy as np
import pytest
import torch

import fused_attn
import oracle
from fused_attn.workloads import make_qkv

TOL_O = {torch.float16: 2e-3, torch.bfloat16: 8e-3}
TOL_LSE = {torch.float16: 1e-3, torch.bfloat16: 1e-3}
REL_CAP = {torch.float16: 1e-2, torch.bfloat16: 5e-2}
THREADS = oracle.default_threads()
N_CASES = 40


def draw(case: int) -> dict:
    rng = random.Random(1000 + case)
    hkv = rng.choice([1, 2, 3, 4])
    return {
        "b": rng.choice([1, 2, 3]),
        "hkv": hkv,
        "h": hkv * rng.choice([1, 2, 4]),
        "n": 32 * rng.randint(1, 40),
        "d": rng.choice([64, 128]),
        "causal": rng.random() < 0.5,
        "dtype": rng.choice([torch.float16, torch.bfloat16]),
        "scale": rng.choice([None, None, round(rng.uniform(0.03, 0.4), 4)]),
        "mag": rng.choice([1.0, 1.0, 2.0]),
        "block_n": rng.choice([0, 0, 64, 128, 32]),
        "strided": rng.random() < 0.3,
        "seed": rng.randint(0, 10**6),
    }


def case_id(case: int) -> str:
    c = draw(case)
    return (f"{case}-B{c['b']}H{c['h']}kv{c['hkv']}N{c['n']}D{c['d']}"
            f"{'c' if c['causal'] else 'f'}-{'bf16' if c['dtype'] == torch.bfloat16 else 'fp16'}"
            f"-bn{c['block_n']}{'-strided' if c['strided'] else ''}")


def unfused_same_dtype(q, k, v, causal, scale):
    """PyTorch's naive attention in the input dtype (the ratio rule's comparison)."""
    h, hkv = q.shape[1], k.shape[1]
    if h != hkv:
        k = k.repeat_interleave(h // hkv, dim=1)
        v = v.repeat_interleave(h // hkv, dim=1)
    s = torch.matmul(q * scale, k.transpose(-1, -2))
    if causal:
        n = q.shape[2]
        s = s.masked_fill(~torch.ones(n, n, dtype=torch.bool, device=q.device).tril(), float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), v)


@pytest.fixture
def reset_overrides():
    yield
    fused_attn.set_debug_overrides(0, 0)


@pytest.mark.gpu
@pytest.mark.parametrize("case", range(N_CASES), ids=case_id)
def test_random_shape_matches_oracle(case, reset_overrides):
    c = draw(case)
    dtype, d = c["dtype"], c["d"]
    if not fused_attn.is_available() or not fused_attn.impl_supports(5, dtype, d):
        pytest.skip("not built for this dtype / head dim")
    q, k, v = make_qkv(c["b"], c["h"], c["n"], d, dtype=dtype, device="cuda", hkv=c["hkv"],
                       seed=c["seed"], scale_inputs=c["mag"])
    fused_attn.set_debug_overrides(0, c["block_n"])
    if c["strided"]:
        # The same values laid out [B, T, H, D] (what a head split of a projection yields).
        qs, ks, vs = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))
        o, lse = fused_attn.forward_strided(qs, ks, vs, is_causal=c["causal"], scale=c["scale"],
                                            return_lse=True)
    else:
        o, lse = fused_attn.forward_stage(q, k, v, 5, is_causal=c["causal"], scale=c["scale"])
    err_dev, bits = fused_attn.last_device_error()
    assert err_dev == 0, f"device status {err_dev} bits={bits:#x}"
    assert bool(torch.isfinite(lse).all()) and bool(torch.isfinite(o).all())
    o_ref, lse_ref = oracle.attention(q, k, v, causal=c["causal"], scale=c["scale"],
                                      threads=THREADS)
    el = oracle.max_abs(lse, lse_ref)
    assert el <= TOL_LSE[dtype], f"max|LSE - LSE_ref| = {el:.3e}"
    ref = np.asarray(o_ref, dtype=np.float64)
    err = np.abs(o.float().cpu().numpy().astype(np.float64) - ref)
    if c["mag"] != 1.0:
        scale = c["scale"] if c["scale"] is not None else 1.0 / d ** 0.5
        r = oracle.error_ratio(o, o_ref, unfused_same_dtype(q, k, v, c["causal"], scale))
        assert r.ok, f"ratio rule failed: {r}"
        assert float(err.max()) <= REL_CAP[dtype] * float(np.abs(ref).max())
        return
    mant = 7 if dtype == torch.bfloat16 else 10
    half_ulp = 0.5 * np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - mant)
    bound = np.maximum(TOL_O[dtype], half_ulp + 2e-3)
    worst = float((err - bound).max())
    assert worst <= 0.0, f"max excess over the bound {worst:.3e} (max|dO| {err.max():.3e})"


def test_draws_cover_every_kernel_and_layout():
    """The 40 draws include every kernel choice, both layouts, GQA, ragged lengths, both dtypes,
    both masks, non-default scales and peaked inputs."""
    cs = [draw(i) for i in range(N_CASES)]
    assert {c["block_n"] for c in cs} == {0, 32, 64, 128}
    assert {c["strided"] for c in cs} == {True, False}
    assert any(c["h"] != c["hkv"] for c in cs)
    assert any(c["n"] % 128 for c in cs)
    assert {c["dtype"] for c in cs} == {torch.float16, torch.bfloat16}
    assert {c["causal"] for c in cs} == {True, False}
    assert any(c["scale"] is not None for c in cs) and any(c["mag"] > 1 for c in cs)


N_CASES_F32 = 12


def draw_f32(case: int) -> dict:
    rng = random.Random(5000 + case)
    hkv = rng.choice([1, 2, 4])
    return {
        "b": rng.choice([1, 2]),
        "hkv": hkv,
        "h": hkv * rng.choice([1, 2]),
        "n": 32 * rng.randint(1, 24),
        "d": rng.choice([64, 128]),
        "causal": rng.random() < 0.5,
        "scale": rng.choice([None, round(rng.uniform(0.03, 0.4), 4)]),
        "strided": rng.random() < 0.3,
        "seed": rng.randint(0, 10**6),
    }


@pytest.mark.gpu
@pytest.mark.parametrize("case", range(N_CASES_F32))
def test_random_fp32_shape_matches_oracle(case):
    """fp32 inputs (tf32 tensor cores after the round-to-nearest pre-pass) on random shapes,
    contiguous or strided: O <= 5e-3 and LSE <= 2e-3 against the oracle (the C1 gates, stated for
    the default scale 1/sqrt(D)).  tf32 keeps 10 explicit mantissa bits of q and k, so a score's
    error is relative to the score: at a softmax scale r times the default the scores, and with them
    the LSE and weight errors, grow r-fold, and both gates are multiplied by max(1, r)."""
    c = draw_f32(case)
    if not fused_attn.is_available() or not fused_attn.impl_supports(3, torch.float32, c["d"]):
        pytest.skip("fp32 path not built")
    q, k, v = make_qkv(c["b"], c["h"], c["n"], c["d"], dtype=torch.float32, device="cuda",
                       hkv=c["hkv"], seed=c["seed"])
    if c["strided"]:
        qs, ks, vs = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))
        o, lse = fused_attn.forward_strided(qs, ks, vs, is_causal=c["causal"], scale=c["scale"],
                                            return_lse=True)
    else:
        o, lse = fused_attn.forward(q, k, v, is_causal=c["causal"], scale=c["scale"],
                                    return_lse=True)
    err_dev, bits = fused_attn.last_device_error()
    assert err_dev == 0, f"device status {err_dev} bits={bits:#x}"
    o_ref, lse_ref = oracle.attention(q, k, v, causal=c["causal"], scale=c["scale"],
                                      threads=THREADS)
    r = 1.0 if c["scale"] is None else max(1.0, c["scale"] * c["d"] ** 0.5)
    assert oracle.max_abs(o, o_ref) <= 5e-3 * r
    assert oracle.max_abs(lse, lse_ref) <= 2e-3 * r
