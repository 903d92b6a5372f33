"""Strided views (``forward_strided`` / ``fa_forward_strided``): the head split and merge of a
GPT-style block without ``.contiguous()`` copies.

No counterpart in the reference, whose op requires contiguous [B, H, N, D] inputs; the results
must equal the contiguous path on the same values (the same kernel reads the same numbers through
a different tensor map), and the oracle gate applies unchanged.
"""

from __future__ import annotations

import math

import pytest
import torch

import fused_attn
import oracle
from fused_attn import abi

pytestmark = pytest.mark.gpu

TOL_O = {torch.float16: 2e-3, torch.bfloat16: 8e-3, torch.float32: 5e-3}
TOL_LSE = {torch.float16: 1e-3, torch.bfloat16: 1e-3, torch.float32: 2e-3}


def require(dtype, d):
    if not fused_attn.is_available():
        pytest.skip("fused_attn._C is not built")
    stage = 3 if dtype == torch.float32 else 5
    if not fused_attn.impl_supports(stage, dtype, d):
        pytest.skip("not built for this device")


def packed_qkv(b, n, h, d, dtype, seed):
    """q, k, v as [B, H, N, D] views of one [B, N, 3, H, D] projection output."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    qkv = torch.randn(b, n, 3, h, d, generator=g).to("cuda", dtype)
    q, k, v = qkv.permute(2, 0, 3, 1, 4)
    return qkv, q, k, v


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("n,d", [(256, 64), (160, 128), (1024, 128)])
def test_packed_projection_views_equal_contiguous(n, d, dtype, causal):
    require(dtype, d)
    b, h = 2, 4
    _, q, k, v = packed_qkv(b, n, h, d, dtype, seed=51)
    assert not q.is_contiguous() and q.stride(3) == 1
    o, lse = fused_attn.forward_strided(q, k, v, is_causal=causal, return_lse=True)
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    o_ref, lse_ref = fused_attn.forward(qc, kc, vc, is_causal=causal, return_lse=True)
    # Same kernel, same numbers: bit-identical to the contiguous path.
    assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref)
    # O has q's layout, so merging heads is a view: [B, H, N, D] -> [B, N, H*D].
    merged = o.transpose(1, 2)
    assert merged.is_contiguous()
    assert merged.reshape(b, n, h * d).data_ptr() == o.data_ptr()
    # And the oracle gate.
    o_or, lse_or = oracle.attention(qc, kc, vc, causal=causal, threads=oracle.default_threads())
    assert oracle.max_abs(o, o_or) <= TOL_O[dtype]
    assert oracle.max_abs(lse, lse_or) <= TOL_LSE[dtype]


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_gqa_separate_q_and_kv_projections(causal):
    require(torch.float16, 128)
    b, n, h, hkv, d = 2, 384, 8, 2, 128
    g = torch.Generator(device="cpu").manual_seed(52)
    xq = torch.randn(b, n, h, d, generator=g).to("cuda", torch.float16)
    xkv = torch.randn(b, n, 2, hkv, d, generator=g).to("cuda", torch.float16)
    q = xq.transpose(1, 2)
    k, v = xkv.permute(2, 0, 3, 1, 4)
    o, lse = fused_attn.forward_strided(q, k, v, is_causal=causal, return_lse=True)
    o_ref, lse_ref = fused_attn.forward(q.contiguous(), k.contiguous(), v.contiguous(),
                                        is_causal=causal, return_lse=True)
    assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref)
    assert o.transpose(1, 2).is_contiguous()


@pytest.mark.parametrize("d", [64, 128])
def test_fp32_strided_views_through_the_rounding_prepass(d):
    require(torch.float32, d)
    b, n, h = 1, 320, 3
    _, q, k, v = packed_qkv(b, n, h, d, torch.float32, seed=53)
    o, lse = fused_attn.forward_strided(q, k, v, is_causal=True, return_lse=True)
    o_ref, lse_ref = fused_attn.forward(q.contiguous(), k.contiguous(), v.contiguous(),
                                        is_causal=True, return_lse=True)
    assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref)


def test_c_abi_padded_strides_and_strided_output():
    """Arbitrary (padded) strides in, a separately strided [B, N, H, D] output buffer out."""
    require(torch.float16, 64)
    b, h, n, d = 2, 3, 192, 64
    g = torch.Generator(device="cpu").manual_seed(54)
    # Each head row padded to 72 elements (144 bytes) and each head to N+8 rows.
    qs = torch.randn(b, h, n + 8, 72, generator=g).to("cuda", torch.float16)
    ks = torch.randn(b, h, n + 8, 72, generator=g).to("cuda", torch.float16)
    vs = torch.randn(b, h, n + 8, 72, generator=g).to("cuda", torch.float16)
    q, k, v = qs[:, :, :n, :d], ks[:, :, :n, :d], vs[:, :, :n, :d]
    out_buf = torch.full((b, n, h, d), float("nan"), device="cuda", dtype=torch.float16)
    o = out_buf.transpose(1, 2)
    lse = torch.full((b, h, n), float("nan"), device="cuda", dtype=torch.float32)
    p = abi.params(b, h, h, n, d, 1.0 / math.sqrt(d), True)
    st = abi.strides(q, k, v, o)
    stream = torch.cuda.current_stream().cuda_stream
    err = abi.forward_strided(abi.FA_IMPL_TUNED, abi.FA_DTYPE_F16, q.data_ptr(), k.data_ptr(),
                              v.data_ptr(), o.data_ptr(), lse.data_ptr(), p, st, stream)
    assert err == 0
    torch.cuda.synchronize()
    o_ref, lse_ref = fused_attn.forward(q.contiguous(), k.contiguous(), v.contiguous(),
                                        is_causal=True, return_lse=True)
    assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref)
    assert fused_attn.last_device_error() == (0, 0)


def test_bad_strides_are_rejected():
    require(torch.float16, 64)
    b, h, n, d = 1, 2, 128, 64
    base = torch.randn(b, h, n, 68, device="cuda", dtype=torch.float16)  # 136-byte rows
    q = base[..., :d]
    k = torch.randn(b, h, n, d, device="cuda", dtype=torch.float16)
    v = torch.randn_like(k)
    with pytest.raises(RuntimeError, match="multiples of 16"):
        fused_attn.forward_strided(q, k, v)
    with pytest.raises(RuntimeError, match="contiguous head dim"):
        fused_attn.forward_strided(k.transpose(2, 3), k, v)
    # The contiguous op keeps the reference's contract.
    with pytest.raises(RuntimeError, match="contiguous"):
        fused_attn.forward(k.transpose(1, 2).contiguous().transpose(1, 2), k, v)
    # C ABI: NULL strides and a bad stride are parameter errors.
    o = torch.empty_like(k)
    lse = torch.empty(b, h, n, device="cuda")
    p = abi.params(b, h, h, n, d, 0.125, False)
    ptrs = (k.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr())
    assert abi.forward_strided(abi.FA_IMPL_TUNED, abi.FA_DTYPE_F16, *ptrs, p, None) == \
        abi.CUDA_ERROR_INVALID_VALUE
    st = abi.strides(k, k, v, o)
    st.k[2] = 68  # 136 bytes
    assert abi.forward_strided(abi.FA_IMPL_TUNED, abi.FA_DTYPE_F16, *ptrs, p, st) == \
        abi.CUDA_ERROR_INVALID_VALUE
