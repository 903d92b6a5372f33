"""Failure detection on the GPU without a GPU fault (marker ``gpu``).

Every mbarrier wait in the kernel is bounded.  Here a wait is made to run out on purpose by a
host-side injection: the producer warp skips the K load of one key tile, so the MMA warp's wait
for it can never complete.  With a 100 ms limit the kernel must record the cause (kStKFull, or
kStKVEmpty when the producer's wait for the slot that tile never frees runs out first), drain its
own copies and MMAs, free its tensor memory and exit normally; the host
reads cudaErrorLaunchTimeout from fa_last_device_error(), and the very next launch on the same
context runs correctly.  No trap, no device assert, no bad address, no endless loop.
"""

from __future__ import annotations

import pytest
import torch

import fused_attn
import oracle

pytestmark = pytest.mark.gpu

K_FULL_BIT = 1 << 1
LAUNCH_TIMEOUT = 702


@pytest.fixture
def restore_knobs():
    yield
    if fused_attn.is_available():
        fused_attn.debug_set_skip_kv_tile(-1)
        fused_attn.set_wait_timeout_ns(2_000_000_000)


KV_EMPTY_BIT = 1 << 6
TOL = {torch.float16: (2e-3, 1e-3), torch.bfloat16: (8e-3, 1e-3), torch.float32: (5e-3, 2e-3)}


@pytest.mark.parametrize("d,dtype,causal", [(64, torch.float16, False), (64, torch.float16, True),
                                            (128, torch.float16, False), (128, torch.bfloat16, False),
                                            (64, torch.float32, False)],
                         ids=["d64-fp16", "d64-fp16-causal-lookahead", "d128-fp16-lookahead",
                              "d128-bf16-lookahead", "d64-fp32-tf32"])
def test_bounded_wait_runs_out_and_context_survives(d, dtype, causal, make_qkv, restore_knobs):
    """Each kernel the dispatcher picks by default (the 128-key kernel for full attention at
    D=64, the lookahead kernel at D=128 and for causal D=64, the tf32 path for fp32).
    Which bounded wait runs out first depends on timing: the MMA issuer's wait for the missing K
    tile (kStKFull) or the producer's wait for the ring slot that tile never frees (kStKVEmpty)."""
    stage = 3 if dtype == torch.float32 else 5
    if not fused_attn.is_available() or not fused_attn.impl_supports(stage, dtype, d):
        pytest.skip("kernel not available")
    q, k, v = make_qkv(1, 2, 512, d, dtype=dtype, device="cuda", seed=41)
    assert fused_attn.last_device_error() == (0, 0)

    fused_attn.set_wait_timeout_ns(100_000_000)
    fused_attn.debug_set_skip_kv_tile(1)
    fused_attn.forward(q, k, v, is_causal=causal)
    err, bits = fused_attn.last_device_error()  # synchronises: the launch has ended
    assert err == LAUNCH_TIMEOUT
    assert bits & (K_FULL_BIT | KV_EMPTY_BIT), f"cause bits {bits:#x}"
    assert fused_attn.last_device_error() == (0, 0)  # read-and-clear

    fused_attn.debug_set_skip_kv_tile(-1)
    fused_attn.set_wait_timeout_ns(2_000_000_000)
    o, lse = fused_attn.forward(q, k, v, is_causal=causal, return_lse=True)
    torch.cuda.synchronize()
    assert fused_attn.last_device_error() == (0, 0)
    o_ref, lse_ref = oracle.attention(q, k, v, causal=causal, threads=oracle.default_threads())
    tol_o, tol_l = TOL[dtype]
    assert oracle.max_abs(o, o_ref) <= tol_o and oracle.max_abs(lse, lse_ref) <= tol_l
