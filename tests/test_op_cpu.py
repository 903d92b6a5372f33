"""CPU checks of the PyTorch operator surface: schemas, fake kernels, wrapper plumbing.

The fakes must give output metadata without running anything (reference
tests/test_op_gpu.py:52-70); under FakeTensorMode no kernel runs, so this needs no GPU.
"""

from __future__ import annotations

import pytest
import torch

import fused_attn

pytestmark = pytest.mark.skipif(not fused_attn.is_available(), reason="fused_attn._C not built")


def test_schemas():
    assert str(torch.ops.fused_attn.forward.default._schema) == (
        "fused_attn::forward(Tensor q, Tensor k, Tensor v, bool is_causal, float scale)"
        " -> (Tensor, Tensor)"
    )
    assert str(torch.ops.fused_attn.forward_stage.default._schema).endswith(
        "int stage) -> (Tensor, Tensor)"
    )


def test_fake_kernels_give_metadata_without_running():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        q = torch.empty(2, 4, 256, 64, dtype=torch.float16, device="cuda")
        k = torch.empty(2, 2, 256, 64, dtype=torch.float16, device="cuda")
        o, lse = torch.ops.fused_attn.forward(q, k, k, False, 0.125)
        assert o.shape == q.shape and o.dtype == q.dtype and o.device.type == "cuda"
        assert lse.shape == (2, 4, 256) and lse.dtype == torch.float32
        for stage in (1, 2, 3, 4, 5):
            o_s, lse_s = torch.ops.fused_attn.forward_stage(q, k, k, True, 0.125, stage)
            assert o_s.shape == q.shape
            assert tuple(lse_s.shape) == ((2, 4, 256) if stage >= 3 else (0,))
        bad = torch.empty(2, 4, 100, 64, dtype=torch.float16, device="cuda")
        with pytest.raises(RuntimeError, match="multiple of 32"):
            torch.ops.fused_attn.forward(bad, bad, bad, False, 0.125)
        bad_d = torch.empty(1, 1, 64, 96, dtype=torch.float16, device="cuda")
        with pytest.raises(RuntimeError, match="D must be 64 or 128"):
            torch.ops.fused_attn.forward(bad_d, bad_d, bad_d, False, 0.125)


def test_cpu_tensors_raise_cuda_message():
    q = torch.randn(1, 2, 64, 64)
    with pytest.raises((RuntimeError, NotImplementedError)):
        fused_attn.forward(q, q, q)


def test_impl_name_op_and_stage_check():
    assert fused_attn.impl_name(5) == "tuned"
    with pytest.raises(RuntimeError, match="stage must be in 1..5"):
        fused_attn.impl_name(0)


def test_default_scale():
    q = torch.empty(1, 1, 32, 128)
    assert fused_attn._resolve_scale(q, None) == pytest.approx(128 ** -0.5)
    assert fused_attn._resolve_scale(q, 0.25) == 0.25
