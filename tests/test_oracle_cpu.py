"""CPU tests that pin the oracle (oracle/fa_oracle.c) before anything is judged against it.

The restatement must reproduce (1) the reference's closed-form known answers
(src/reference/test_cpu_reference.cpp:39-67), (2) the reference's own compiled oracle
(oracle/_ref, built from src/reference/cpu_reference.cpp where it lies) bit for bit,
(3) the golden fixtures that the reference's two oracles produced (tests/golden/gen_golden.py),
and (4) the properties the reference tests: tiled == direct for any tiling, scale folding,
sum_j exp(s_ij - lse_i) == 1, causal == explicit tril mask, guard behaviour.  A recurrence with a
planted bug must fail the tile-invariance check (tests/test_reference_cpu.py:258-302 "teeth").
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN_DIR

TOL64 = 1e-12


def qkv64(b, h, n, d, seed=0, hkv=None):
    from fused_attn.workloads import make_qkv

    return make_qkv(b, h, n, d, dtype=torch.float64, hkv=hkv, seed=seed)


def lcg_fill(shape, seed):
    """Deterministic [-1, 1) values (a 64-bit LCG, as the reference's ctest uses)."""
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float64)
    mask = (1 << 64) - 1
    st = (seed * 6364136223846793005 + 1442695040888963407) & mask
    for i in range(n):
        st = (st * 6364136223846793005 + 1442695040888963407) & mask
        out[i] = (st >> 11) * (1.0 / 9007199254740992.0) * 2.0 - 1.0
    return out.reshape(shape)


# ------------------------------------------------------------------------------------------
# 1. Closed-form known answers: q = k = I2, v = [[1, 2], [3, 4]], scale = 1.
# ------------------------------------------------------------------------------------------
def test_known_answer_2x2():
    q = np.array([[[[1.0, 0.0], [0.0, 1.0]]]])
    v = np.array([[[[1.0, 2.0], [3.0, 4.0]]]])
    e = math.e
    o, lse = oracle.attention(q, q, v, causal=False, scale=1.0)
    want = np.array([[(e * 1 + 3) / (1 + e), (e * 2 + 4) / (1 + e)],
                     [(1 + 3 * e) / (1 + e), (2 + 4 * e) / (1 + e)]])
    assert np.abs(o[0, 0] - want).max() < 1e-14
    assert np.abs(lse[0, 0] - math.log(1 + e)).max() < 1e-14
    o, lse = oracle.attention(q, q, v, causal=True, scale=1.0)
    assert o[0, 0, 0, 0] == 1.0 and o[0, 0, 0, 1] == 2.0  # row 0 sees key 0 only
    assert abs(lse[0, 0, 0] - 1.0) < 1e-15
    assert np.abs(o[0, 0, 1] - want[1]).max() < 1e-14
    assert abs(lse[0, 0, 1] - math.log(1 + e)) < 1e-14


# ------------------------------------------------------------------------------------------
# 2. The restatement equals the reference's own compiled oracle.
# ------------------------------------------------------------------------------------------
needs_ref = pytest.mark.skipif(not oracle.ref_available(),
                               reason="oracle/_ref not built (make -C oracle ref)")


@needs_ref
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("b,h,hkv,n,d", [(1, 2, 2, 128, 64), (2, 4, 2, 96, 128), (1, 3, 1, 64, 64)])
def test_restatement_equals_reference_oracle(b, h, hkv, n, d, causal):
    q, k, v = qkv64(b, h, n, d, seed=3, hkv=hkv)
    o, lse = oracle.attention(q, k, v, causal=causal, threads=4)
    o_r, lse_r, _ = oracle.ref_attention(q, k, v, causal=causal, threads=4)
    assert np.array_equal(o, o_r)
    assert np.array_equal(lse, lse_r)
    o_t, lse_t = oracle.tiled(q, k, v, 32, 16, causal=causal)
    o_rt, lse_rt = oracle.ref_tiled(q, k, v, 32, 16, causal=causal)
    assert np.array_equal(o_t, o_rt) and np.array_equal(lse_t, lse_rt)


@needs_ref
def test_rows_equal_reference_rows():
    q, k, v = qkv64(2, 4, 40, 16, seed=7, hkv=2)
    o, lse = oracle.rows(q, k, v, 1, 3, 5, 7, causal=True, scale=0.25)
    o_r, lse_r = oracle.ref_rows(q, k, v, 1, 3, 5, 7, causal=True, scale=0.25)
    assert np.array_equal(o, o_r) and np.array_equal(lse, lse_r)


def test_reference_ctest_passes_when_built():
    import subprocess

    exe = oracle.HERE / "_ref" / "test_cpu_reference"
    if not exe.exists():
        pytest.skip("reference ctest not built (make -C oracle ref)")
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=False)
    assert out.returncode == 0 and "PASS" in out.stdout


# ------------------------------------------------------------------------------------------
# 3. Golden fixtures produced by the reference's two oracles.
# ------------------------------------------------------------------------------------------
def _golden():
    return np.load(GOLDEN_DIR / "golden.npz")


def golden_cases():
    with _golden() as g:
        return sorted({k.split("/")[0] for k in g.files})


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("name", golden_cases())
def test_oracle_matches_golden(name, causal):
    g = _golden()
    b, h, hkv, n, d, seed, dt = (int(x) for x in g[f"{name}/meta"])
    scale = float(g[f"{name}/scale"][0])
    scale = None if math.isnan(scale) else scale
    q, k, v = (g[f"{name}/{t}"] for t in ("q", "k", "v"))
    assert q.shape == (b, h, n, d) and k.shape == (b, hkv, n, d)
    tag = "causal" if causal else "full"
    o, lse = oracle.attention(q, k, v, causal=causal, scale=scale)
    assert oracle.max_abs(o, g[f"{name}/{tag}/o"]) < TOL64
    assert oracle.max_abs(lse, g[f"{name}/{tag}/lse"]) < TOL64


def test_golden_inputs_follow_the_seeded_generator():
    """The fixtures' inputs are exactly what make_qkv(seed) produces (so GPU tests can
    regenerate them on the device side and compare with the stored expectations)."""
    from fused_attn.workloads import make_qkv

    g = _golden()
    for name in golden_cases():
        b, h, hkv, n, d, seed, dt = (int(x) for x in g[f"{name}/meta"])
        dtype = {0: torch.float32, 1: torch.float16, 2: torch.bfloat16}[dt]
        q, k, v = make_qkv(b, h, n, d, dtype=dtype, hkv=hkv, seed=seed)
        for t, tn in ((q, "q"), (k, "k"), (v, "v")):
            assert np.array_equal(t.float().numpy(), g[f"{name}/{tn}"].astype(np.float32)), (name, tn)


# ------------------------------------------------------------------------------------------
# 4. Properties (test_cpu_reference.cpp:69-136, test_reference_cpu.py).
# ------------------------------------------------------------------------------------------
@pytest.mark.parametrize("n,d,h,hkv", [(64, 64, 4, 2), (96, 32, 2, 2), (40, 128, 4, 1)])
def test_tiled_equals_direct(n, d, h, hkv):
    q = lcg_fill((2, h, n, d), 1)
    k = lcg_fill((2, hkv, n, d), 2)
    v = lcg_fill((2, hkv, n, d), 3)
    for causal in (False, True):
        o_ref, lse_ref = oracle.attention(q, k, v, causal=causal)
        for bm, bn in [(n, n), (32, 16), (16, 8), (8, 64), (64, 8), (1, 1), (n, 7)]:
            o, lse = oracle.tiled(q, k, v, bm, bn, causal=causal)
            assert oracle.max_abs(o, o_ref) < TOL64, (causal, bm, bn)
            assert oracle.max_abs(lse, lse_ref) < 1e-11, (causal, bm, bn)


def test_causal_tile_skip_is_exact():
    q, k, v = qkv64(1, 2, 128, 64)
    a = oracle.tiled(q, k, v, 32, 16, causal=True, skip_masked=True)
    b = oracle.tiled(q, k, v, 32, 16, causal=True, skip_masked=False)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_scale_folding_and_lse_normalisation():
    q, k, v = qkv64(2, 4, 40, 16, seed=7, hkv=2)
    o, lse = oracle.attention(q, k, v, causal=True, scale=0.25)
    o2, lse2 = oracle.attention(q * 2, k, v, causal=True, scale=0.125)
    assert oracle.max_abs(o, o2) < 1e-13 and oracle.max_abs(lse, lse2) < 1e-12
    # sum_j exp(scale * q_i . k_j - lse_i) == 1 over visible keys
    qn, kn = q.numpy(), k.numpy()
    kr = np.repeat(kn, 2, axis=1)
    s = np.einsum("bhid,bhjd->bhij", qn, kr) * 0.25
    s = np.where(np.tril(np.ones((40, 40), dtype=bool)), s, -np.inf)
    tot = np.exp(s - lse[..., None]).sum(-1)
    assert np.abs(tot - 1.0).max() < 1e-12


def test_numpy_restatement_agrees():
    q, k, v = qkv64(2, 2, 64, 64, seed=4)
    for causal in (False, True):
        o, lse = oracle.attention(q, k, v, causal=causal)
        o_n, lse_n = oracle.numpy_attention(q, k, v, causal=causal)
        assert oracle.max_abs(o, o_n) < 1e-12 and oracle.max_abs(lse, lse_n) < 1e-12


def test_causal_equals_tril_mask_and_row0_is_v0():
    q, k, v = qkv64(1, 2, 128, 64, seed=4)
    o_c, lse_c = oracle.attention(q, k, v, causal=True)
    o_m, lse_m = oracle.numpy_attention(q, k, v, keep=np.tril(np.ones((128, 128), dtype=bool)))
    assert oracle.max_abs(o_c, o_m) < 1e-12 and oracle.max_abs(lse_c, lse_m) < 1e-12
    assert oracle.max_abs(o_c[:, :, 0], v[:, :, 0]) < 1e-15


def test_fully_masked_rows_give_zero_and_posinf():
    q, k, v = qkv64(1, 1, 16, 8, seed=5)
    keep = np.ones((16, 16), dtype=bool)
    keep[5, :] = False
    o, lse = oracle.numpy_attention(q, k, v, keep=keep)
    assert np.all(o[0, 0, 5] == 0) and np.isposinf(lse[0, 0, 5])
    assert np.isfinite(o).all()


def _tiled_with_planted_bug(q, k, v, block_n, bug):
    """Copy of the recurrence with one step removed -- the mistake is planted here, in the
    CPU model, never in GPU code.  bug: 'no_acc_rescale' or 'no_l_rescale'."""
    q, k, v = (np.asarray(t, dtype=np.float64) for t in (q, k, v))
    b, h, n, d = q.shape
    c = (1.0 / math.sqrt(d)) * oracle.LOG2E
    m = np.full((b, h, n, 1), -np.inf)
    l = np.zeros((b, h, n, 1))
    acc = np.zeros((b, h, n, d))
    for j0 in range(0, n, block_n):
        s = np.einsum("bhid,bhjd->bhij", q, k[:, :, j0:j0 + block_n])
        m_new = np.maximum(m, s.max(-1, keepdims=True))
        alpha = np.exp2((m - m_new) * c)
        p = np.exp2((s - m_new) * c)
        l = (l if bug == "no_l_rescale" else alpha * l) + p.sum(-1, keepdims=True)
        acc = (acc if bug == "no_acc_rescale" else alpha * acc) + p @ v[:, :, j0:j0 + block_n]
        m = m_new
    return acc / l


@pytest.mark.parametrize("bug", ["no_acc_rescale", "no_l_rescale"])
def test_planted_rescale_bug_is_caught(bug):
    q, k, v = qkv64(1, 2, 128, 64, seed=9)
    o_ref, _ = oracle.attention(q, k, v)
    assert oracle.max_abs(_tiled_with_planted_bug(q, k, v, 128, bug), o_ref) < 1e-12
    assert oracle.max_abs(_tiled_with_planted_bug(q, k, v, 32, bug), o_ref) > 1e-3


def test_error_ratio_rule():
    g = np.random.default_rng(6)
    ref = g.standard_normal((2, 2, 32, 64))
    noise = g.standard_normal(ref.shape)
    same = ref + 1e-3 * noise
    good = oracle.error_ratio(ref + 1e-3 * noise[::-1], ref, same)
    assert good.ok and good.err_mine <= good.bound
    assert not oracle.error_ratio(ref + 1e-2 * noise, ref, same).ok
    bad = ref.copy()
    bad[0, 0, 0, 0] = np.nan
    assert not oracle.error_ratio(bad, ref, same).out_finite


def test_threaded_oracle_is_deterministic():
    q, k, v = qkv64(2, 3, 96, 64, seed=11)
    a = oracle.attention(q, k, v, causal=True, threads=1)
    b = oracle.attention(q, k, v, causal=True, threads=7)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
