"""GPU parity of the sm_100a kernel against the CPU oracle (marker ``gpu``).

Reference counterpart: tests/test_kernels_gpu.py.  Gate, per output element, against the fp64
oracle run on the very (rounded) inputs the kernel saw:

    fp16: max|O - O_ref| <= 2e-3 and max|LSE - LSE_ref| <= 1e-3
    bf16: max|O - O_ref| <= 8e-3 and max|LSE - LSE_ref| <= 1e-3

plus the reference's secondary FlashAttention ratio rule (error <= 2x PyTorch's own unfused
attention in the same dtype + 1e-6) and its absolute caps.  Every BASELINE configuration is
checked over the whole tensor against the oracle, the C3 sweep up to N=8192 included; C4 (32
heads of N=16384) over two whole heads, sampled rows of others (as the reference's fa_bench
self-check samples tiles), and the whole tensor against PyTorch's fp32 SDPA as an extra opinion.
Head-sharded runs (what each GPU of the multi-GPU configuration computes) must equal the
one-launch result bit for bit.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import fused_attn
import oracle
from conftest import GOLDEN_DIR
from fused_attn import abi
from fused_attn.workloads import C3_SWEEP_N, CONFIGS

pytestmark = pytest.mark.gpu

DTYPES = [torch.float16, torch.bfloat16]
TOL_O = {torch.float16: 2e-3, torch.bfloat16: 8e-3}
TOL_LSE = {torch.float16: 1e-3, torch.bfloat16: 1e-3}
ABS_CAP = {torch.float16: 1e-2, torch.bfloat16: 5e-2}
_ids = {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32"}
THREADS = oracle.default_threads()


def dtype_id(dt):
    return _ids[dt]


def require(dtype=torch.float16, d=64):
    if not fused_attn.is_available():
        pytest.skip("fused_attn._C is not built")
    if not fused_attn.impl_supports(5, dtype, d):
        cap = torch.cuda.get_device_capability()
        pytest.skip(f"not built for {_ids[dtype]} D={d} on sm_{cap[0]}{cap[1]}")


@pytest.fixture
def reset_overrides():
    yield
    if fused_attn.is_available():
        fused_attn.set_debug_overrides(0, 0)


def unfused_same_dtype(q, k, v, causal, scale=None):
    """PyTorch's naive attention in the input dtype (reference.py:288-311): the ratio term."""
    h, hkv = q.shape[1], k.shape[1]
    if h != hkv:
        k = k.repeat_interleave(h // hkv, dim=1)
        v = v.repeat_interleave(h // hkv, dim=1)
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    s = torch.matmul(q * scale, k.transpose(-1, -2))
    if causal:
        n = q.shape[2]
        s = s.masked_fill(~torch.ones(n, n, dtype=torch.bool, device=q.device).tril(), float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), v)


def check(o, lse, q, k, v, causal, dtype, scale=None, ratio=True):
    """Full-tensor gate against the oracle.  Returns (err_o, err_lse)."""
    assert o.shape == q.shape and o.dtype == dtype and o.is_contiguous()
    assert lse.shape == q.shape[:3] and lse.dtype == torch.float32
    assert bool(torch.isfinite(o).all()), "kernel produced NaN/inf"
    assert bool(torch.isfinite(lse).all())
    o_ref, lse_ref = oracle.attention(q, k, v, causal=causal, scale=scale, threads=THREADS)
    eo = oracle.max_abs(o, o_ref)
    el = oracle.max_abs(lse, lse_ref)
    assert eo <= TOL_O[dtype], f"max|O - O_ref| = {eo:.3e} > {TOL_O[dtype]}"
    assert el <= TOL_LSE[dtype], f"max|LSE - LSE_ref| = {el:.3e} > {TOL_LSE[dtype]}"
    if ratio:
        r = oracle.error_ratio(o, o_ref, unfused_same_dtype(q, k, v, causal, scale))
        assert r.ok, f"ratio rule failed: {r}"
        assert r.err_mine <= ABS_CAP[dtype]
    return eo, el


def check_rows(o, lse, q, k, v, causal, dtype, row_blocks, scale=None):
    """Oracle on selected (b, h, row0, nrows) blocks only (large configs)."""
    o_c, lse_c = o.float().cpu(), lse.cpu()
    qc, kc, vc = q.cpu(), k.cpu(), v.cpu()
    for b, h, r0, nr in row_blocks:
        o_ref, lse_ref = oracle.rows(qc, kc, vc, b, h, r0, nr, causal=causal, scale=scale)
        eo = oracle.max_abs(o_c[b, h, r0:r0 + nr], o_ref)
        el = oracle.max_abs(lse_c[b, h, r0:r0 + nr], lse_ref)
        assert eo <= TOL_O[dtype], f"rows {(b, h, r0, nr)}: max|dO| = {eo:.3e}"
        assert el <= TOL_LSE[dtype], f"rows {(b, h, r0, nr)}: max|dLSE| = {el:.3e}"


def check_vs_sdpa_fp32(o, q, k, v, causal, dtype):
    """Whole-tensor comparison against PyTorch fp32 SDPA (a floating-point reference of the
    same op, on the same rounded inputs), for configs too large for the oracle."""
    import torch.nn.functional as F

    h, hkv = q.shape[1], k.shape[1]
    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal,
                                         enable_gqa=h != hkv)
    err = float((o.float() - ref).abs().max())
    assert err <= TOL_O[dtype], f"max|O - SDPA_fp32| = {err:.3e}"


def sample_blocks(b, h, n, tile=128):
    mid = (n // 2 // tile) * tile
    starts = sorted({0, mid, max(0, n - tile)})
    return [(bb, hh, r0, min(tile, n - r0)) for bb, hh in {(0, 0), (b - 1, h - 1)} for r0 in starts]


# ------------------------------------------------------------------------------------------
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("dtype", DTYPES, ids=dtype_id)
def test_matches_oracle(dtype, causal, gpu_shape, make_qkv):
    b, h, n, d = gpu_shape
    require(dtype, d)
    q, k, v = make_qkv(b, h, n, d, dtype=dtype, device="cuda")
    o, lse = fused_attn.forward_stage(q, k, v, 5, is_causal=causal)
    check(o, lse, q, k, v, causal, dtype)


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("n", [32, 96, 160, 224, 416])
def test_ragged_sequence_lengths(n, d, causal, make_qkv):
    """N % 32 == 0 but not a multiple of the 128-row tile: partial query and key tiles."""
    require(torch.float16, d)
    q, k, v = make_qkv(2, 3, n, d, dtype=torch.float16, device="cuda", seed=21)
    o, lse = fused_attn.forward(q, k, v, is_causal=causal, return_lse=True)
    check(o, lse, q, k, v, causal, torch.float16)


@pytest.mark.parametrize("name", ["C2", "C2c", "C3", "C3bf16"])
def test_baseline_configs(name, make_qkv):
    cfg = CONFIGS[name]
    require(cfg.dtype, cfg.D)
    q, k, v = make_qkv(cfg.B, cfg.H, cfg.N, cfg.D, dtype=cfg.dtype, device="cuda", seed=cfg.seed)
    o, lse = fused_attn.forward(q, k, v, is_causal=cfg.causal, return_lse=True)
    check(o, lse, q, k, v, cfg.causal, cfg.dtype, ratio=False)


@pytest.mark.parametrize("dtype", DTYPES, ids=dtype_id)
@pytest.mark.parametrize("n", C3_SWEEP_N)
def test_c3_sequence_sweep(n, dtype, make_qkv):
    require(dtype, 128)
    q, k, v = make_qkv(2, 8, n, 128, dtype=dtype, device="cuda", seed=2)
    o, lse = fused_attn.forward(q, k, v, is_causal=True, return_lse=True)
    # The whole tensor against the oracle at every N (N=8192: ~9 s of fp64 on 16 host threads).
    check(o, lse, q, k, v, True, dtype, ratio=False)
    if n >= 4096:
        check_vs_sdpa_fp32(o, q, k, v, True, dtype)


def test_c4_long_context(make_qkv):
    """C4 (B1 H32 N16384 D128 bf16 causal, seed 3) on one GPU: two whole heads (the first and
    the last) against the oracle, sampled rows of two more, and the whole tensor against fp32
    SDPA."""
    cfg = CONFIGS["C4"]
    require(cfg.dtype, cfg.D)
    q, k, v = make_qkv(cfg.B, cfg.H, cfg.N, cfg.D, dtype=cfg.dtype, device="cuda", seed=cfg.seed)
    o, lse = fused_attn.forward(q, k, v, is_causal=True, return_lse=True)
    assert bool(torch.isfinite(o).all()) and bool(torch.isfinite(lse).all())
    for h in (0, cfg.H - 1):
        sl = slice(h, h + 1)
        check(o[:, sl].contiguous(), lse[:, sl].contiguous(), q[:, sl].contiguous(),
              k[:, sl].contiguous(), v[:, sl].contiguous(), True, cfg.dtype, ratio=False)
    blocks = [(0, 17, cfg.N // 2, 64), (0, 9, cfg.N - 32, 32)]
    check_rows(o, lse, q, k, v, True, cfg.dtype, blocks)
    check_vs_sdpa_fp32(o, q, k, v, True, cfg.dtype)


@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_head_shards_equal_one_launch_bitwise(ranks, make_qkv):
    """What each GPU of the head-sharded configuration computes (a contiguous block of H/ranks
    heads, as fused_attn.sharding assigns them) equals the same heads of one launch over all
    heads, bit for bit: a head's result does not depend on which other heads share the launch
    or on how the persistent CTAs were dealt the work."""
    from fused_attn import sharding

    require(torch.bfloat16, 128)
    b, h, n, d = 1, 32, 2048, 128
    q, k, v = make_qkv(b, h, n, d, dtype=torch.bfloat16, device="cuda", seed=3)
    o, lse = fused_attn.forward(q, k, v, is_causal=True, return_lse=True)
    for r in range(ranks):
        h0, h1 = sharding.head_range(h, ranks, r)
        qs, ks, vs = (t[:, h0:h1].contiguous() for t in (q, k, v))
        o_r, lse_r = fused_attn.forward(qs, ks, vs, is_causal=True, return_lse=True)
        assert torch.equal(o_r, o[:, h0:h1]) and torch.equal(lse_r, lse[:, h0:h1]), r


# ------------------------------------------------------------------------------------------
@pytest.mark.parametrize("dtype", DTYPES, ids=dtype_id)
@pytest.mark.parametrize("name", ["fp16_n64", "bf16_n96_d128", "fp16_scale005_d128"])
def test_golden_fixtures(name, dtype):
    """The kernel against outputs the reference's own oracles produced (tests/golden)."""
    g = np.load(GOLDEN_DIR / "golden.npz")
    b, h, hkv, n, d, seed, dt = (int(x) for x in g[f"{name}/meta"])
    want_dtype = {1: torch.float16, 2: torch.bfloat16}.get(dt)
    if want_dtype != dtype:
        pytest.skip("fixture stored for the other dtype")
    require(dtype, d)
    scale = float(g[f"{name}/scale"][0])
    scale = None if math.isnan(scale) else scale
    q, k, v = (torch.from_numpy(g[f"{name}/{t}"].astype(np.float32)).to("cuda", dtype) for t in "qkv")
    for causal in (False, True):
        tag = "causal" if causal else "full"
        o, lse = fused_attn.forward(q, k, v, is_causal=causal, scale=scale, return_lse=True)
        eo = oracle.max_abs(o, g[f"{name}/{tag}/o"])
        el = oracle.max_abs(lse, g[f"{name}/{tag}/lse"])
        assert eo <= TOL_O[dtype] and el <= TOL_LSE[dtype], (tag, eo, el)


# ------------------------------------------------------------------------------------------
def test_forward_dispatches_to_stage5(make_qkv):
    require()
    q, k, v = make_qkv(1, 2, 256, 64, dtype=torch.float16, device="cuda")
    o, lse = fused_attn.forward(q, k, v, is_causal=True, return_lse=True)
    o5, lse5 = fused_attn.forward_stage(q, k, v, 5, is_causal=True)
    assert torch.equal(o, o5) and torch.equal(lse, lse5)


@pytest.mark.parametrize("n", [128, 256])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("dtype", DTYPES, ids=dtype_id)
def test_tile_invariance(dtype, causal, n, make_qkv, reset_overrides):
    """The online-softmax rescale only runs when a row spans several key tiles: the same
    problem with block_n in {128, 64, 32} must pass the gate every time and agree."""
    require(dtype, 64)
    q, k, v = make_qkv(2, 2, n, 64, dtype=dtype, device="cuda", seed=11)
    outs = {}
    for bm, bn in [(0, 0), (0, 64), (0, 32), (128, 32)]:
        fused_attn.set_debug_overrides(bm, bn)
        o, lse = fused_attn.forward_stage(q, k, v, 5, is_causal=causal)
        torch.cuda.synchronize()
        check(o, lse, q, k, v, causal, dtype)
        outs[(bm, bn)] = o.double()
    fused_attn.set_debug_overrides(0, 0)
    base = outs[(0, 0)]
    for key, o in outs.items():
        assert float((o - base).abs().max()) <= 2 * TOL_O[dtype], key


def test_unbuilt_tile_override_is_rejected(make_qkv, reset_overrides):
    require()
    q, k, v = make_qkv(1, 1, 128, 64, dtype=torch.float16, device="cuda")
    for bm, bn in [(64, 0), (0, 48), (0, 256)]:
        fused_attn.set_debug_overrides(bm, bn)
        with pytest.raises(RuntimeError, match="invalid argument"):
            fused_attn.forward(q, k, v)
    fused_attn.set_debug_overrides(0, 0)


@pytest.mark.parametrize("dtype", DTYPES, ids=dtype_id)
def test_determinism_50_runs_bitwise_equal(dtype, make_qkv):
    require(dtype, 64)
    q, k, v = make_qkv(2, 4, 256, 64, dtype=dtype, device="cuda", seed=12)
    first, first_lse = fused_attn.forward_stage(q, k, v, 5, is_causal=True)
    for _ in range(49):
        o, lse = fused_attn.forward_stage(q, k, v, 5, is_causal=True)
        assert torch.equal(o, first) and torch.equal(lse, first_lse)


@pytest.mark.parametrize("factor", [1e2, 1e-3], ids=["x1e2", "x1e-3"])
@pytest.mark.parametrize("dtype", DTYPES, ids=dtype_id)
def test_half_precision_dynamic_range(dtype, factor, make_qkv):
    """Scores past fp16's range must stay in fp32 (x1e2); tiny scores (x1e-3)."""
    require(dtype, 64)
    q, k, v = make_qkv(1, 2, 256, 64, dtype=dtype, device="cuda", seed=13, scale_inputs=factor)
    o, lse = fused_attn.forward_stage(q, k, v, 5)
    assert bool(torch.isfinite(o).all()) and bool(torch.isfinite(lse).all())
    o_ref, lse_ref = oracle.attention(q, k, v, threads=THREADS)
    rel = oracle.max_abs(o, o_ref) / max(float(np.abs(o_ref).max()), 1e-30)
    assert rel <= ABS_CAP[dtype]
    assert oracle.max_abs(lse, lse_ref) <= max(TOL_LSE[dtype], 1e-6 * float(np.abs(lse_ref).max()))


@pytest.mark.parametrize("dtype", DTYPES, ids=dtype_id)
def test_causal_equals_explicit_tril_mask(dtype, make_qkv):
    require(dtype, 64)
    n = 512
    q, k, v = make_qkv(1, 2, n, 64, dtype=dtype, device="cuda", seed=14)
    o, _ = fused_attn.forward_stage(q, k, v, 5, is_causal=True)
    o_mask, _ = oracle.numpy_attention(q, k, v, keep=np.tril(np.ones((n, n), dtype=bool)))
    assert oracle.max_abs(o, o_mask) <= TOL_O[dtype]
    # query 0 sees key 0 only: o[0] == v[0] exactly (v[0] is representable in the dtype)
    assert torch.equal(o[:, :, 0, :], v[:, :, 0, :])


@pytest.mark.parametrize("bn", [64, 128], ids=["lookahead", "kt128"])
@pytest.mark.parametrize("n", [128, 160])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", DTYPES, ids=dtype_id)
def test_many_short_items_per_cta(dtype, d, causal, n, bn, make_qkv, reset_overrides):
    """768 / 1536 one- or two-round items on 148 CTAs: five to eleven item epilogues per CTA back
    to back, so the exchange and O staging buffers, the O_free hand-off and the first item's loads
    issued from the prologue are all exercised many times per CTA (N=160 adds a ragged tile)."""
    require(dtype, d)
    q, k, v = make_qkv(16, 48, n, d, dtype=dtype, device="cuda", seed=23)
    fused_attn.set_debug_overrides(0, bn)
    o, lse = fused_attn.forward_stage(q, k, v, 5, is_causal=causal)
    o_ref, lse_ref = oracle.attention(q, k, v, causal=causal, threads=THREADS)
    assert oracle.max_abs(lse, lse_ref) <= TOL_LSE[dtype]
    # Over 768 heads some causal rows average only 1-3 keys and reach |O| >= 4, where a single
    # bf16 rounding of the exact result is already up to 2^-6 = 1.56e-2 (PyTorch's own bf16
    # attention misses by 1.7e-2 on these inputs).  So each element must meet the dtype's gate or,
    # where larger, half a unit in the last place of its reference value in the output dtype plus
    # 2e-3.
    ref = np.asarray(o_ref, dtype=np.float64)
    err = np.abs(o.float().cpu().numpy().astype(np.float64) - ref)
    mant = 7 if dtype == torch.bfloat16 else 10
    half_ulp = 0.5 * np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - mant)
    bound = np.maximum(TOL_O[dtype], half_ulp + 2e-3)
    worst = float((err - bound).max())
    assert worst <= 0.0, f"max excess over the bound {worst:.3e} (max|dO| {err.max():.3e})"


@pytest.mark.parametrize("bn", [0, 64, 128], ids=["default", "lookahead", "kt128"])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", DTYPES, ids=dtype_id)
def test_running_max_jumps_in_late_key_tiles(dtype, d, causal, bn, make_qkv, reset_overrides):
    """Keys whose scores jump far above every earlier score of their rows (a query-aligned key
    scaled by 6) in the third and fifth key tiles: the running max of those rows rises by far more
    than the lazy-rescale threshold mid-item, so the O correction of a later tile runs (fp16's
    lazy path and bf16's eager one), in every kernel."""
    require(dtype, d)
    q, k, v = make_qkv(1, 2, 640, d, dtype=dtype, device="cuda", seed=19)
    for pos in (300, 531):
        k[:, :, pos, :] = q[:, :, pos + 7, :] * 6
    fused_attn.set_debug_overrides(0, bn)
    o, lse = fused_attn.forward_stage(q, k, v, 5, is_causal=causal)
    check(o, lse, q, k, v, causal, dtype)


@pytest.mark.parametrize("scale", [0.05, 0.25])
@pytest.mark.parametrize("dtype", DTYPES, ids=dtype_id)
def test_non_default_scale(dtype, scale, make_qkv):
    require(dtype, 128)
    q, k, v = make_qkv(1, 2, 256, 128, dtype=dtype, device="cuda", seed=15)
    o, lse = fused_attn.forward_stage(q, k, v, 5, is_causal=False, scale=scale)
    check(o, lse, q, k, v, False, dtype, scale=scale)


@pytest.mark.parametrize("h,hkv", [(4, 2), (8, 1), (6, 3)])
@pytest.mark.parametrize("dtype", DTYPES, ids=dtype_id)
def test_gqa_heads(dtype, h, hkv, make_qkv):
    require(dtype, 64)
    q, k, v = make_qkv(2, h, 256, 64, dtype=dtype, device="cuda", hkv=hkv, seed=17)
    o, lse = fused_attn.forward_stage(q, k, v, 5, is_causal=True)
    check(o, lse, q, k, v, True, dtype)


# ------------------------------------------------------------------------------------------
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_c_abi_direct_call_equals_op_and_overwrites_poison(causal, make_qkv):
    """fa_forward through ctypes on caller-owned, NaN-poisoned buffers on torch's current
    stream: every O/LSE element is written and equals the op's result bit for bit."""
    require()
    b, h, n, d = 2, 3, 352, 128
    q, k, v = make_qkv(b, h, n, d, dtype=torch.float16, device="cuda", seed=31)
    o = torch.full_like(q, float("nan"))
    lse = torch.full((b, h, n), float("nan"), device="cuda", dtype=torch.float32)
    p = abi.params(b, h, h, n, d, 1.0 / math.sqrt(d), causal)
    stream = torch.cuda.current_stream().cuda_stream
    err = abi.forward(abi.FA_IMPL_TUNED, abi.FA_DTYPE_F16, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                      o.data_ptr(), lse.data_ptr(), p, stream)
    assert err == 0
    torch.cuda.synchronize()
    assert bool(torch.isfinite(o).all()) and bool(torch.isfinite(lse).all())
    o_op, lse_op = fused_attn.forward(q, k, v, is_causal=causal, return_lse=True)
    assert torch.equal(o, o_op) and torch.equal(lse, lse_op)
    assert fused_attn.last_device_error() == (0, 0)


def test_c_abi_error_codes_on_device(make_qkv):
    require()
    q, k, v = make_qkv(1, 2, 128, 64, dtype=torch.float16, device="cuda")
    o, lse = torch.empty_like(q), torch.empty(1, 2, 128, device="cuda")
    ptrs = (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr())
    p = abi.params(1, 2, 2, 128, 64, 0.125, False)
    assert abi.forward(abi.FA_IMPL_WMMA, abi.FA_DTYPE_F16, *ptrs, p) == abi.CUDA_ERROR_NOT_SUPPORTED
    assert abi.forward(abi.FA_IMPL_TUNED, abi.FA_DTYPE_F32, *ptrs, p) == abi.CUDA_ERROR_NOT_SUPPORTED
    p.N = 100
    assert abi.forward(abi.FA_IMPL_TUNED, abi.FA_DTYPE_F16, *ptrs, p) == abi.CUDA_ERROR_INVALID_VALUE


# ------------------------------------------------------------------------------------------
def test_n_not_multiple_of_32_raises(make_qkv):
    require()
    q, k, v = make_qkv(1, 1, 100, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 32"):
        fused_attn.forward_stage(q, k, v, 5)
    with pytest.raises(RuntimeError, match="multiple of 32"):
        fused_attn.forward(q, k, v)


def test_input_validation_messages(make_qkv):
    require()
    q, k, v = make_qkv(1, 2, 64, 64, dtype=torch.float16, device="cuda")
    with pytest.raises((RuntimeError, NotImplementedError)):
        fused_attn.forward(q.cpu(), k.cpu(), v.cpu())
    with pytest.raises(RuntimeError, match="contiguous"):
        fused_attn.forward(q.transpose(1, 2).contiguous().transpose(1, 2), k, v)
    with pytest.raises(RuntimeError, match="dtype"):
        fused_attn.forward(q, k.float(), v)
    with pytest.raises(RuntimeError, match="D must be 64 or 128"):
        fused_attn.forward(q[..., :32].contiguous(), k[..., :32].contiguous(),
                           v[..., :32].contiguous())
    with pytest.raises(RuntimeError, match="stage must be in 1..5"):
        fused_attn.forward_stage(q, k, v, 0)
    with pytest.raises(RuntimeError, match="stage must be in 1..5"):
        fused_attn.forward_stage(q, k, v, 6)
    with pytest.raises(RuntimeError, match="Nq == Nkv"):
        fused_attn.forward(q, k[:, :, :32].contiguous(), v[:, :, :32].contiguous())
    with pytest.raises(RuntimeError, match="multiple of Hkv"):
        fused_attn.forward(q[:, :1].contiguous(), k, v)
    with pytest.raises(RuntimeError, match="16-byte aligned"):
        flat = torch.empty(64 * 64 * 2 + 1, dtype=torch.float16, device="cuda")
        qm = flat[1:].view(1, 2, 64, 64)
        fused_attn.forward(qm, k, v)
    with pytest.raises(RuntimeError, match="scale must be finite"):
        fused_attn.forward(q, k, v, scale=0.0)
    for stage in (1, 2, 4):
        with pytest.raises(RuntimeError, match="not implemented"):
            fused_attn.forward_stage(q, k, v, stage)
    with pytest.raises(RuntimeError, match="not implemented|no stage"):
        fused_attn.forward_stage(q.float(), k.float(), v.float(), 5)


# ------------------------------------------------------------------------------------------
def test_launch_past_2_31_elements():
    """Maximum sizes: q, k, v and o of B65 H16 N16384 D128 fp16 (causal) hold 2.18e9 elements
    each, so the last heads sit past element offset 2^31 and any 32-bit offset in the tensor
    maps, the O stores or the LSE index would misplace them.  The first and the last head of the
    one 17 GB launch equal one-head launches of the same inputs bit for bit (a head's result does
    not depend on the launch it is in), and the last head matches the oracle on sampled rows
    (converted to fp64 on the host one head at a time: the whole tensor would not fit)."""
    require(torch.float16, 128)
    b, h, n, d = 65, 16, 16384, 128
    assert b * h * n * d > 2 ** 31
    need = 4 * b * h * n * d * 2 + b * h * n * 4
    free, _ = torch.cuda.mem_get_info()
    if free < need + (4 << 30):
        pytest.skip(f"needs {need / 2**30:.1f} GiB of device memory, {free / 2**30:.1f} free")
    try:
        _check_large_launch(b, h, n, d)
    finally:
        torch.cuda.empty_cache()


def _check_large_launch(b, h, n, d):
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (torch.randn(b, h, n, d, device="cuda", dtype=torch.float16, generator=g)
               for _ in range(3))
    o, lse = fused_attn.forward(q, k, v, is_causal=True, return_lse=True)
    torch.cuda.synchronize()
    err, bits = fused_attn.last_device_error()
    assert err == 0, f"device status {err} bits={bits:#x}"
    assert bool(torch.isfinite(lse[-1, -1]).all()) and bool(torch.isfinite(o[-1, -1]).all())
    for bb, hh in ((b - 1, h - 1), (0, 0)):
        qs, ks, vs = (t[bb:bb + 1, hh:hh + 1].contiguous() for t in (q, k, v))
        o1, l1 = fused_attn.forward(qs, ks, vs, is_causal=True, return_lse=True)
        assert torch.equal(o1, o[bb:bb + 1, hh:hh + 1]), (bb, hh)
        assert torch.equal(l1, lse[bb:bb + 1, hh:hh + 1]), (bb, hh)
    last = slice(b - 1, b), slice(h - 1, h)
    qc, kc, vc = (t[last].cpu() for t in (q, k, v))
    blocks = [(0, 0, 0, 64), (0, 0, n // 2, 64), (0, 0, n - 64, 64)]
    check_rows(o[last], lse[last], qc, kc, vc, True, torch.float16, blocks)
