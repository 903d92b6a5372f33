"""PyTorch custom-op conformance on the GPU (marker ``gpu``).

Reference counterpart: tests/test_op_gpu.py -- ``torch.library.opcheck`` on both ops, the
fake kernels, ``torch.compile(fullgraph=True)`` with zero graph breaks and a bitwise-equal
result, dynamic sequence length, and the Python wrapper against the raw op.
"""

from __future__ import annotations

import pytest
import torch

import fused_attn
from fused_attn import ops
from fused_attn.ops import opcheck_all

pytestmark = pytest.mark.gpu

DTYPES = [torch.float16, torch.bfloat16]


def require(dtype=torch.float16, d=64):
    if not fused_attn.is_available():
        pytest.skip("fused_attn._C is not built")
    if not fused_attn.impl_supports(5, dtype, d):
        pytest.skip("stage 5 not built for this device")


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("dtype", DTYPES, ids=["fp16", "bf16"])
def test_opcheck_all_ops(dtype, causal, make_qkv):
    require(dtype)
    q, k, v = make_qkv(1, 2, 64, 64, dtype=dtype, device="cuda")
    results = opcheck_all(q, k, v, is_causal=causal, stages=[5])
    assert set(results) == {"forward", "forward_strided", "forward_stage[5]"}
    for name, res in results.items():
        assert all(status in ("SUCCESS", "SKIPPED") for status in res.values()), (name, res)


def test_opcheck_strided_op_on_views():
    """opcheck of forward_strided on non-contiguous head-split views (fake kernel = real layout)."""
    require(torch.float16, 64)
    x = torch.randn(1, 64, 3, 2, 64, device="cuda", dtype=torch.float16)
    q, k, v = x.permute(2, 0, 3, 1, 4)
    res = ops._opcheck(torch.ops.fused_attn.forward_strided, (q, k, v, True, 0.125))
    assert all(status in ("SUCCESS", "SKIPPED") for status in res.values()), res


def test_compile_fullgraph_gpt_head_split_without_copies():
    """torch.compile(fullgraph=True) of split-heads -> forward_strided -> merge-heads."""
    require(torch.float16, 64)
    b, t, h, d = 2, 128, 4, 64

    def block(qkv):
        q, k, v = qkv.view(b, t, 3, h, d).permute(2, 0, 3, 1, 4)
        o = fused_attn.forward_strided(q, k, v, is_causal=True)
        return o.transpose(1, 2).reshape(b, t, h * d)

    x = torch.randn(b, t, 3 * h * d, device="cuda", dtype=torch.float16)
    eager = block(x)
    compiled = torch.compile(block, fullgraph=True)(x)
    assert torch.equal(eager, compiled)


@pytest.mark.parametrize("dtype", DTYPES, ids=["fp16", "bf16"])
def test_torch_compile_fullgraph_no_graph_break(dtype, make_qkv):
    require(dtype)
    q, k, v = make_qkv(1, 2, 128, 64, dtype=dtype, device="cuda")

    def f(q, k, v):
        q = q * 1.0
        o, lse = torch.ops.fused_attn.forward(q, k, v, True, 0.125)
        return o * 2.0, lse + 1.0

    torch._dynamo.reset()
    explanation = torch._dynamo.explain(f)(q, k, v)
    assert explanation.graph_break_count == 0, explanation.break_reasons
    assert explanation.graph_count == 1

    torch._dynamo.reset()
    from torch._dynamo.utils import counters

    counters.clear()
    compiled = torch.compile(f, fullgraph=True)
    out = compiled(q, k, v)
    assert sum(counters["graph_break"].values()) == 0
    ref = f(q, k, v)
    torch.testing.assert_close(out[0], ref[0], atol=0, rtol=0)
    torch.testing.assert_close(out[1], ref[1], atol=0, rtol=0)


def test_torch_compile_dynamic_shapes_forward_stage(make_qkv):
    """Dynamic N: the fake's torch._check(N % 32 == 0) must become a guard, not a break."""
    require()

    def g(q, k, v):
        o, lse = torch.ops.fused_attn.forward_stage(q, k, v, False, 0.125, 5)
        return o.float().sum(-1), lse

    torch._dynamo.reset()
    compiled = torch.compile(g, fullgraph=True, dynamic=True)
    for n in (128, 256, 384):
        q, k, v = make_qkv(1, 2, n, 64, dtype=torch.float16, device="cuda")
        o_sum, lse = compiled(q, k, v)
        ref_sum, ref_lse = g(q, k, v)
        torch.testing.assert_close(o_sum, ref_sum, atol=1e-3, rtol=1e-3)
        assert lse.shape == ref_lse.shape


def test_public_wrapper_matches_raw_op(make_qkv):
    require()
    q, k, v = make_qkv(1, 2, 64, 64, dtype=torch.float16, device="cuda")
    o_wrap = fused_attn.forward(q, k, v, is_causal=True)  # default scale 1/sqrt(64)
    o_raw, lse_raw = torch.ops.fused_attn.forward(q, k, v, True, 0.125)
    assert torch.equal(o_wrap, o_raw)
    o2, lse2 = fused_attn.forward(q, k, v, is_causal=True, return_lse=True)
    assert torch.equal(o2, o_raw) and torch.equal(lse2, lse_raw)
    assert fused_attn.impl_name(5) == "tuned"


def test_op_runs_on_a_side_stream(make_qkv):
    """The op launches on torch's current stream (no implicit sync, no default stream)."""
    require()
    q, k, v = make_qkv(2, 2, 512, 128, dtype=torch.float16, device="cuda", seed=3)
    ref = fused_attn.forward(q, k, v, is_causal=True)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        o = fused_attn.forward(q, k, v, is_causal=True)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    assert torch.equal(o, ref)


def test_cuda_graph_capture_replays(make_qkv):
    """The launch is capturable: no host sync and no allocation inside fa_forward."""
    require()
    q, k, v = make_qkv(2, 4, 256, 64, dtype=torch.float16, device="cuda", seed=4)
    ref = fused_attn.forward(q, k, v, is_causal=True)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fused_attn.forward(q, k, v, is_causal=True)  # warm-up on the capture stream
        with torch.cuda.graph(g, stream=s):
            out = fused_attn.forward(q, k, v, is_causal=True)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
