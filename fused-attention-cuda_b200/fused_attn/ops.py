"""Fake (meta) kernels and the opcheck helper for the ``fused_attn::*`` ops.

Reference counterpart: python/fused_attn/ops.py.  ``torch.compile`` traces ops on fake tensors;
without a fake kernel a ``TORCH_LIBRARY`` op is a graph break.  The fakes below mirror the
TORCH_CHECKs of csrc/ext.cpp with ``torch._check`` so they hold under symbolic shapes, and
return the output metadata: ``forward`` -> (O like q, LSE [B, H, N] fp32).
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
from torch import Tensor

SUPPORTED_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
SUPPORTED_HEAD_DIMS = (64, 128)
LSE_STAGES = (3, 4, 5)

_registered = False


def _check_inputs(q: Tensor, k: Tensor, v: Tensor) -> None:
    torch._check(q.dim() == 4 and k.dim() == 4 and v.dim() == 4, lambda: "q/k/v must be [B,H,N,D]")
    torch._check(q.dtype == k.dtype and q.dtype == v.dtype, lambda: "q/k/v must share one dtype")
    torch._check(q.dtype in SUPPORTED_DTYPES, lambda: f"unsupported dtype {q.dtype}")
    b, h, n, d = q.shape
    torch._check(d == 64 or d == 128, lambda: f"D must be 64 or 128, got {d}")
    torch._check(n % 32 == 0, lambda: f"N must be a multiple of 32, got {n}")
    torch._check(k.shape[0] == b and v.shape[0] == b, lambda: "batch mismatch")
    torch._check(k.shape[2] == n and v.shape[2] == n, lambda: "Nq == Nkv is required in-window")
    torch._check(k.shape[3] == d and v.shape[3] == d, lambda: "head-dim mismatch")
    torch._check(k.shape[1] == v.shape[1], lambda: "k and v must have the same number of heads")
    torch._check(h % k.shape[1] == 0, lambda: "H must be a multiple of Hkv")


def _fake_forward(q: Tensor, k: Tensor, v: Tensor, is_causal: bool, scale: float):
    _check_inputs(q, k, v)
    b, h, n, _ = q.shape
    return torch.empty_like(q), q.new_empty((b, h, n), dtype=torch.float32)


def _fake_forward_strided(q: Tensor, k: Tensor, v: Tensor, is_causal: bool, scale: float):
    # O takes q's layout (empty_like keeps a dense view's strides), LSE is contiguous.
    _check_inputs(q, k, v)
    b, h, n, _ = q.shape
    return torch.empty_like(q), q.new_empty((b, h, n), dtype=torch.float32)


def _fake_combine(o_parts, lse_parts):
    torch._check(len(o_parts) >= 1 and len(o_parts) == len(lse_parts),
                 lambda: "combine needs as many LSE tensors as O partials")
    o0 = o_parts[0]
    b, h, n, _ = o0.shape
    return torch.empty_like(o0, memory_format=torch.contiguous_format), \
        o0.new_empty((b, h, n), dtype=torch.float32)


def _fake_forward_stage(q: Tensor, k: Tensor, v: Tensor, is_causal: bool, scale: float, stage: int):
    _check_inputs(q, k, v)
    torch._check(1 <= stage <= 5, lambda: f"stage must be in 1..5, got {stage}")
    b, h, n, _ = q.shape
    o = torch.empty_like(q)
    if stage in LSE_STAGES:
        lse = q.new_empty((b, h, n), dtype=torch.float32)
    else:
        lse = q.new_empty((0,), dtype=torch.float32)
    return o, lse


def register_fakes() -> None:
    """Register the fake kernels (idempotent; needs ``fused_attn._C`` loaded)."""
    global _registered
    if _registered:
        return
    torch.library.register_fake("fused_attn::forward", _fake_forward)
    torch.library.register_fake("fused_attn::forward_stage", _fake_forward_stage)
    torch.library.register_fake("fused_attn::forward_strided", _fake_forward_strided)
    torch.library.register_fake("fused_attn::combine", _fake_combine)
    _registered = True


# torch.library.opcheck utilities and the inputs each must see.  The ops have no autograd kernel:
# test_autograd_registration is meant to run on tensors that require grad (it checks that such a
# call is not silently differentiable), while the schema / fake-tensor / AOT-dispatch utilities
# must see plain tensors.  (The reference's ops.py splits its opcheck the same way, for the same
# reason: the split follows from opcheck's own contract.)
_OPCHECK_PLAN = (
    (("test_schema", "test_faketensor", "test_aot_dispatch_dynamic"), False),
    (("test_autograd_registration",), True),
)


def _grad_inputs(args: tuple, on: bool) -> tuple:
    """`args` with every floating-point tensor detached and requiring grad when `on`."""
    if not on:
        return args
    return tuple(a.detach().requires_grad_() if isinstance(a, Tensor) and a.is_floating_point()
                 else a for a in args)


def _opcheck(op, args: tuple) -> dict[str, str]:
    report: dict[str, str] = {}
    for utils, grad in _OPCHECK_PLAN:
        report.update(torch.library.opcheck(op, _grad_inputs(args, grad), test_utils=utils))
    return report


def opcheck_all(q: Tensor, k: Tensor, v: Tensor, is_causal: bool = False,
                scale: float | None = None, stages: Sequence[int] = ()) -> dict[str, dict[str, str]]:
    """``torch.library.opcheck`` on ``forward`` and on ``forward_stage`` for each stage."""
    if scale is None:
        scale = 1.0 / (q.shape[-1] ** 0.5)
    results: dict[str, dict[str, str]] = {}
    results["forward"] = _opcheck(torch.ops.fused_attn.forward, (q, k, v, is_causal, float(scale)))
    results["forward_strided"] = _opcheck(torch.ops.fused_attn.forward_strided,
                                          (q, k, v, is_causal, float(scale)))
    for stage in stages:
        results[f"forward_stage[{stage}]"] = _opcheck(
            torch.ops.fused_attn.forward_stage, (q, k, v, is_causal, float(scale), int(stage))
        )
    return results
