"""fp32 inputs: the tf32 tensor-core flavour of the kernel, served as stage 3 ("fused").

Reference counterpart: the fp32 rows of tests/test_kernels_gpu.py, which run the reference's
fa_s3_fused (src/stage3_fused.cu, fp32 FFMA).  On B200 the same recurrence runs on tcgen05
kind::tf32: Q, K, V enter the tensor core with a 10-bit mantissa (the fp16 mantissa, fp32
exponent range) and P is rounded to tf32 before the P V product; the softmax, the running sums
and the accumulators stay fp32.  Gate against the fp64 oracle on the fp32 inputs, stated for
tf32 operands:

    max|O - O_ref| <= 5e-3,  max|LSE - LSE_ref| <= 2e-3.

The reference's ratio rule (error <= 2x an unfused fp32 computation) does not apply: it assumes
fp32 arithmetic, which tf32 operands are not.
"""

from __future__ import annotations

import math

import pytest
import torch

import fused_attn
import oracle
from fused_attn import abi
from fused_attn.workloads import CONFIGS

pytestmark = pytest.mark.gpu

TOL_O_TF32 = 5e-3
TOL_LSE_TF32 = 2e-3
THREADS = oracle.default_threads()


def require(d=64):
    if not fused_attn.is_available():
        pytest.skip("fused_attn._C is not built")
    if not fused_attn.impl_supports(3, torch.float32, d):
        cap = torch.cuda.get_device_capability()
        pytest.skip(f"fp32 D={d} is not built for sm_{cap[0]}{cap[1]}")


@pytest.fixture
def reset_overrides():
    yield
    if fused_attn.is_available():
        fused_attn.set_debug_overrides(0, 0)


def check_tf32(o, lse, q, k, v, causal, scale=None):
    assert o.shape == q.shape and o.dtype == torch.float32 and o.is_contiguous()
    assert lse.shape == q.shape[:3] and lse.dtype == torch.float32
    assert bool(torch.isfinite(o).all()) and bool(torch.isfinite(lse).all())
    o_ref, lse_ref = oracle.attention(q, k, v, causal=causal, scale=scale, threads=THREADS)
    eo = oracle.max_abs(o, o_ref)
    el = oracle.max_abs(lse, lse_ref)
    assert eo <= TOL_O_TF32, f"max|O - O_ref| = {eo:.3e} > {TOL_O_TF32}"
    assert el <= TOL_LSE_TF32, f"max|LSE - LSE_ref| = {el:.3e} > {TOL_LSE_TF32}"
    return eo, el


@pytest.mark.parametrize("name", ["C1", "C1c"])
def test_c1_fp32_config(name, make_qkv):
    """C1 (B1 H2 N128 D64 fp32, seed 0): the reference's CPU-runnable configuration."""
    cfg = CONFIGS[name]
    require(cfg.D)
    q, k, v = make_qkv(cfg.B, cfg.H, cfg.N, cfg.D, dtype=torch.float32, device="cuda", seed=cfg.seed)
    o, lse = fused_attn.forward(q, k, v, is_causal=cfg.causal, return_lse=True)
    check_tf32(o, lse, q, k, v, cfg.causal)


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("b,h,n,d", [(1, 1, 32, 64), (2, 3, 96, 128), (2, 3, 352, 128),
                                     (1, 2, 1024, 64), (2, 2, 1024, 128)])
def test_fp32_matches_oracle(b, h, n, d, causal, make_qkv):
    require(d)
    q, k, v = make_qkv(b, h, n, d, dtype=torch.float32, device="cuda", seed=41)
    o, lse = fused_attn.forward_stage(q, k, v, 3, is_causal=causal)
    check_tf32(o, lse, q, k, v, causal)


def test_forward_picks_stage3_for_fp32(make_qkv):
    require()
    q, k, v = make_qkv(1, 2, 256, 64, dtype=torch.float32, device="cuda", seed=42)
    o, lse = fused_attn.forward(q, k, v, is_causal=True, return_lse=True)
    o3, lse3 = fused_attn.forward_stage(q, k, v, 3, is_causal=True)
    assert torch.equal(o, o3) and torch.equal(lse, lse3)
    with pytest.raises(RuntimeError, match="not implemented"):
        fused_attn.forward_stage(q, k, v, 5, is_causal=True)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_fp32_tile_invariance(causal, d, make_qkv, reset_overrides):
    require(d)
    q, k, v = make_qkv(2, 2, 320, d, dtype=torch.float32, device="cuda", seed=43)
    outs = []
    for bn in ([0, 32, 64, 128] if d == 64 else [0, 32, 64]):
        fused_attn.set_debug_overrides(0, bn)
        o, lse = fused_attn.forward_stage(q, k, v, 3, is_causal=causal)
        torch.cuda.synchronize()
        check_tf32(o, lse, q, k, v, causal)
        outs.append(o.double())
    for o in outs[1:]:
        assert float((o - outs[0]).abs().max()) <= 2 * TOL_O_TF32


@pytest.mark.parametrize("h,hkv", [(4, 2), (6, 1)])
def test_fp32_gqa(h, hkv, make_qkv):
    require(128)
    q, k, v = make_qkv(2, h, 256, 128, dtype=torch.float32, device="cuda", hkv=hkv, seed=44)
    o, lse = fused_attn.forward(q, k, v, is_causal=True, return_lse=True)
    check_tf32(o, lse, q, k, v, True)


def test_fp32_values_beyond_half_range(make_qkv):
    """V scaled by 1e6 (past fp16's 65504): tf32 keeps fp32's exponent range, so O stays
    within the same relative gate; LSE does not depend on V."""
    require(64)
    q, k, v = make_qkv(1, 2, 256, 64, dtype=torch.float32, device="cuda", seed=45)
    v = v * 1e6
    o, lse = fused_attn.forward(q, k, v, is_causal=True, return_lse=True)
    assert bool(torch.isfinite(o).all()) and bool(torch.isfinite(lse).all())
    o_ref, lse_ref = oracle.attention(q, k, v, causal=True, threads=THREADS)
    assert oracle.max_abs(o, o_ref) <= TOL_O_TF32 * 1e6
    assert oracle.max_abs(lse, lse_ref) <= TOL_LSE_TF32


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_fp32_c_abi_direct_call(causal, make_qkv):
    """fa_forward(Impl::Fused, fp32) on caller-owned NaN-poisoned buffers equals the op."""
    require(128)
    b, h, n, d = 2, 2, 288, 128
    q, k, v = make_qkv(b, h, n, d, dtype=torch.float32, device="cuda", seed=46)
    o = torch.full_like(q, float("nan"))
    lse = torch.full((b, h, n), float("nan"), device="cuda", dtype=torch.float32)
    p = abi.params(b, h, h, n, d, 1.0 / math.sqrt(d), causal)
    stream = torch.cuda.current_stream().cuda_stream
    ptrs = (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr())
    ws_bytes = abi.workspace_bytes(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, p)
    assert ws_bytes == 3 * q.numel() * 4
    # The workspace is required: NULL is a parameter error, reported before any launch.
    assert abi.forward(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, *ptrs, p, stream) == \
        abi.CUDA_ERROR_INVALID_VALUE
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    err = abi.forward(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, *ptrs, p, stream, ws.data_ptr())
    assert err == 0
    torch.cuda.synchronize()
    o_op, lse_op = fused_attn.forward(q, k, v, is_causal=causal, return_lse=True)
    assert torch.equal(o, o_op) and torch.equal(lse, lse_op)
    assert fused_attn.last_device_error() == (0, 0)
