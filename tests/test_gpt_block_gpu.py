"""GPT-2 block harness on the GPU (marker ``gpu``): the C5 workload through our op.

Reference counterpart: bench/gpt_block.py.  The strided call (no ``.contiguous()`` copies) and
the reference's contiguous call run the same kernel on the same numbers, so the block outputs
must be bit-identical; the attention itself is gated against PyTorch's fp32 math attention with
the fp16 kernel gate (2e-3), and the whole block against PyTorch SDPA in fp16.
"""

from __future__ import annotations

import pytest
import torch

import fused_attn
from fused_attn import gpt_block as gb

pytestmark = pytest.mark.gpu

CFG = gb.GPTConfig(batch=2)  # GPT-2-small block at T=1024, batch 2 for the test


def require():
    if not fused_attn.is_available():
        pytest.skip("fused_attn._C is not built")
    if not fused_attn.impl_supports(5, torch.float16, 64):
        pytest.skip("not built for this device")


def test_strided_and_contiguous_calls_are_bit_identical():
    require()
    ids = gb.token_ids(CFG, "cuda")
    with torch.no_grad():
        a = gb.build_model(CFG, "fused_strided", "cuda")(ids)
        b = gb.build_model(CFG, "fused_contiguous", "cuda")(ids)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert fused_attn.last_device_error() == (0, 0)


def test_attention_matches_fp32_math_and_block_matches_sdpa():
    require()
    ids = gb.token_ids(CFG, "cuda")
    ours = gb.build_model(CFG, "fused_strided", "cuda")
    ref = gb.build_model(CFG, "sdpa_math", "cuda")
    with torch.no_grad():
        x = ours.block.ln_1(ours.wte(ids) + ours.wpe(torch.arange(CFG.seq, device="cuda")))
        b, t, c = x.shape
        q, k, v = ours.block.attn.c_attn(x).view(b, t, 3, CFG.n_head, CFG.head_dim).permute(2, 0, 3, 1, 4)
        o = ours.block.attn.attend(q, k, v)
        o32 = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                                               is_causal=True)
        assert float((o.float() - o32).abs().max()) <= 2e-3
        y, y_ref = ours(ids), ref(ids)
    err = float((y.float() - y_ref.float()).abs().max())
    assert err <= 2e-3 * (1.0 + float(y_ref.float().abs().max())), err


def test_measure_reports_tokens_per_second():
    require()
    cfg = gb.GPTConfig(batch=1, seq=256)
    model = gb.build_model(cfg, "fused_strided", "cuda")
    m = gb.measure(model, gb.token_ids(cfg, "cuda"), warmup=2, iters=5)
    assert m["block_ms"] > 0 and m["attn_ms"] > 0 and 0 < m["attn_pct"] < 100
    assert m["tokens_per_s"] == pytest.approx(256 / (m["block_ms"] * 1e-3))
    assert m["block_ms_p10"] <= m["block_ms"] <= m["block_ms_p90"]
