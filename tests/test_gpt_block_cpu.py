"""GPT-2 block harness (fused_attn/gpt_block.py, config C5) on the CPU.

Reference counterpart: bench/gpt_block.py.  Checks what needs no GPU: the C5 FLOP counts, the
seeded initialisation (identical across attention impls), the head split and merge being views
for the strided path, the block running end to end with PyTorch's math attention, and the fused
impls refusing CPU tensors instead of falling back.
"""

from __future__ import annotations

import pytest
import torch

from fused_attn import gpt_block as gb

SMALL = gb.GPTConfig(n_embd=128, n_head=2, seq=64, batch=2, dtype=torch.float32)


def test_c5_flop_counts():
    cfg = gb.GPTConfig()
    assert cfg.head_dim == 64
    assert cfg.attention_flops() == pytest.approx(25.77e9, rel=1e-3)
    assert cfg.gemm_flops() == pytest.approx(231.9e9, rel=1e-3)


def test_initialisation_is_seeded_and_impl_independent():
    a = gb.build_model(SMALL, "sdpa_math", "cpu")
    b = gb.build_model(SMALL, "fused_strided", "cpu")
    for (na, pa), (nb, pb) in zip(a.named_parameters(), b.named_parameters(), strict=True):
        assert na == nb and torch.equal(pa, pb), na
    assert float(a.block.ln_1.weight.detach().min()) == 1.0
    assert float(a.block.attn.c_attn.bias.detach().abs().max()) == 0.0
    assert 0.015 < float(a.wte.weight.detach().std()) < 0.025
    ids = gb.token_ids(SMALL, "cpu")
    assert ids.shape == (2, 64) and int(ids.min()) >= 0 and int(ids.max()) < gb.VOCAB
    assert torch.equal(ids, gb.token_ids(SMALL, "cpu"))


def test_head_split_is_a_view_of_the_projection():
    b, t, h, d = 2, 16, 4, 8
    qkv = torch.randn(b, t, 3 * h * d)
    q, k, v = qkv.view(b, t, 3, h, d).permute(2, 0, 3, 1, 4)
    for x in (q, k, v):
        assert x.shape == (b, h, t, d) and x.stride(-1) == 1
        assert x.untyped_storage().data_ptr() == qkv.untyped_storage().data_ptr()
    # an output laid out like q's dense order ([B, T, H, D]) merges heads without a copy
    o = torch.empty(b, t, h, d).transpose(1, 2)
    merged = o.transpose(1, 2).reshape(b, t, h * d)
    assert merged.data_ptr() == o.data_ptr()


def test_block_runs_with_math_attention_and_matches_manual_attention():
    model = gb.build_model(SMALL, "sdpa_math", "cpu")
    ids = gb.token_ids(SMALL, "cpu")
    with torch.no_grad():
        y = model(ids)
        # the same block with attention written out by hand
        blk = model.block
        x = model.wte(ids) + model.wpe(torch.arange(SMALL.seq))
        hx = blk.ln_1(x)
        qkv = blk.attn.c_attn(hx)
        b, t, c = hx.shape
        q, k, v = qkv.view(b, t, 3, SMALL.n_head, SMALL.head_dim).permute(2, 0, 3, 1, 4)
        s = (q @ k.transpose(-1, -2)) * blk.attn.scale
        s = s.masked_fill(~torch.ones(t, t, dtype=torch.bool).tril(), float("-inf"))
        a = (s.softmax(-1) @ v).transpose(1, 2).reshape(b, t, c)
        x = x + blk.attn.c_proj(a)
        ref = x + blk.mlp(blk.ln_2(x))
    assert y.shape == (2, 64, 128)
    assert float((y - ref).abs().max()) < 1e-5


@pytest.mark.parametrize("impl", gb.FUSED_IMPLS)
def test_fused_impls_refuse_cpu_tensors(impl):
    import fused_attn

    if not fused_attn.is_available():
        pytest.skip("fused_attn._C is not built")
    model = gb.build_model(SMALL, impl, "cpu")
    with pytest.raises((RuntimeError, NotImplementedError)):
        with torch.no_grad():
            model(gb.token_ids(SMALL, "cpu"))


def test_unknown_impl_is_rejected():
    with pytest.raises(ValueError, match="unknown attention impl"):
        gb.CausalSelfAttention(SMALL, "sdpa_magic")
