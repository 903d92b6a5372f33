"""Split-KV combine on the GPU (``fa_combine`` / ``torch.ops.fused_attn.combine``).

* the kernel against ``oracle.combine`` on random partials with "no key" sentinel rows;
* ring / context-parallel causal attention: a sequence split into S chunks, chunk c attends to
  chunks 0..c with the forward (the diagonal chunk top-left causal) and the partials are merged;
  the result must pass the forward's oracle gate on the unsplit problem, with the tolerance
  doubled (each partial carries its own rounding, the merge adds the output rounding once);
* non-causal key splits; fp32 partials; the C ABI's parameter errors.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fused_attn
import oracle
from fused_attn import abi
from fused_attn.workloads import make_qkv

pytestmark = pytest.mark.gpu

TOL_O = {torch.float16: 2e-3, torch.bfloat16: 8e-3, torch.float32: 5e-3}
TOL_LSE = {torch.float16: 1e-3, torch.bfloat16: 1e-3, torch.float32: 2e-3}


def require():
    if not fused_attn.is_available():
        pytest.skip("fused_attn._C is not built")
    if not fused_attn.impl_supports(5, torch.float16, 64):
        pytest.skip("not built for this device")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32],
                         ids=["fp16", "bf16", "fp32"])
@pytest.mark.parametrize("d", [64, 128])
def test_kernel_matches_oracle_with_sentinels(d, dtype):
    require()
    g = torch.Generator(device="cpu").manual_seed(71)
    s, b, h, n = 5, 2, 3, 96
    o_parts = [torch.randn(b, h, n, d, generator=g).to("cuda", dtype) for _ in range(s)]
    lse_parts = [(torch.randn(b, h, n, generator=g) * 3).cuda() for _ in range(s)]
    # Rows with no keys in some partials (+inf and -inf), and a row with none anywhere.
    lse_parts[1][0, 0, :10] = float("inf")
    lse_parts[3][1, 2, 5:9] = float("-inf")
    for p in lse_parts:
        p[1, 1, 7] = float("inf")
    o, lse = fused_attn.combine(o_parts, lse_parts)
    o_ref, lse_ref = oracle.combine(o_parts, lse_parts)
    assert o.dtype == dtype and o.shape == (b, h, n, d) and lse.dtype == torch.float32
    # One rounding of the output: half an ulp, relative 2^-11 (fp16) / 2^-8 (bf16); doubled.
    rel = {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7, torch.float32: 1e-6}[dtype]
    assert oracle.max_abs(o, o_ref) <= rel * max(1.0, float(np.abs(o_ref).max()))
    finite = np.isfinite(lse_ref)
    assert np.abs(lse.cpu().numpy()[finite] - lse_ref[finite]).max() <= 1e-5
    assert float(lse[1, 1, 7]) == float("inf") and bool((o[1, 1, 7] == 0).all())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("d", [64, 128])
def test_ring_causal_attention_from_chunks(d, dtype):
    """Causal self-attention over 4 chunks of 256 tokens, assembled from per-chunk forwards."""
    require()
    b, h, n, s = 1, 2, 1024, 4
    q, k, v = make_qkv(b, h, n, d, dtype=dtype, device="cuda", seed=72)
    qs, ks, vs = (list(t.chunk(s, dim=2)) for t in (q, k, v))
    qs, ks, vs = ([c.contiguous() for c in t] for t in (qs, ks, vs))
    o_full, lse_full = oracle.attention(q, k, v, causal=True, threads=oracle.default_threads())
    cl = n // s
    for c in range(s):
        parts = [fused_attn.forward(qs[c], ks[j], vs[j], is_causal=(j == c), return_lse=True)
                 for j in range(c + 1)]
        o, lse = fused_attn.combine([p[0] for p in parts], [p[1] for p in parts])
        rows = slice(c * cl, (c + 1) * cl)
        assert oracle.max_abs(o, o_full[:, :, rows]) <= 2 * TOL_O[dtype], c
        assert oracle.max_abs(lse, lse_full[:, :, rows]) <= TOL_LSE[dtype], c


def test_noncausal_key_split_fp32():
    require()
    if not fused_attn.impl_supports(3, torch.float32, 64):
        pytest.skip("fp32 not built")
    b, h, n, d, s = 1, 2, 512, 64, 4
    q, k, v = make_qkv(b, h, n, d, dtype=torch.float32, device="cuda", seed=73)
    qs, ks, vs = ([c.contiguous() for c in t.chunk(s, dim=2)] for t in (q, k, v))
    o_full, lse_full = oracle.attention(q, k, v, causal=False, threads=oracle.default_threads())
    cl = n // s
    for c in range(s):
        parts = [fused_attn.forward(qs[c], ks[j], vs[j], return_lse=True) for j in range(s)]
        o, lse = fused_attn.combine([p[0] for p in parts], [p[1] for p in parts])
        rows = slice(c * cl, (c + 1) * cl)
        assert oracle.max_abs(o, o_full[:, :, rows]) <= 2 * TOL_O[torch.float32]
        assert oracle.max_abs(lse, lse_full[:, :, rows]) <= TOL_LSE[torch.float32]


def test_parameter_errors():
    require()
    o = torch.zeros(1, 1, 32, 64, device="cuda", dtype=torch.float16)
    lse = torch.zeros(1, 1, 32, device="cuda")
    with pytest.raises(RuntimeError, match="as many LSE"):
        fused_attn.combine([o, o], [lse])
    with pytest.raises(RuntimeError, match="at most"):
        fused_attn.combine([o] * (abi.COMBINE_MAX_SPLITS + 1), [lse] * (abi.COMBINE_MAX_SPLITS + 1))
    out = torch.empty_like(o)
    lo = torch.empty_like(lse)
    args = (out.data_ptr(), lo.data_ptr(), 1, 1, 32, 64)
    assert abi.combine(abi.FA_DTYPE_F16, [], [], *args) == abi.CUDA_ERROR_INVALID_VALUE
    assert abi.combine(abi.FA_DTYPE_F16, [o.data_ptr()], [lse.data_ptr()], out.data_ptr(),
                       lo.data_ptr(), 1, 1, 32, 96) == abi.CUDA_ERROR_INVALID_VALUE
    assert abi.combine(abi.FA_DTYPE_F16, [o.data_ptr()], [lse.data_ptr()], *args) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, o) and torch.equal(lo, lse)
