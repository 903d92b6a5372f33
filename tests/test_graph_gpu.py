"""The op inside a CUDA graph (marker ``gpu``).

No counterpart in the reference.  A launch-bound caller (a decode loop, a small block) captures
the forward into a CUDA graph; the op launches only on the current stream, allocates only
through PyTorch's caching allocator (fp32's workspace included) and never synchronises, so
capture works and every replay must reproduce the eager result bit for bit.
"""

from __future__ import annotations

import pytest
import torch

import fused_attn
from fused_attn.workloads import make_qkv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("d,dtype,causal", [(128, torch.float16, True), (64, torch.float16, False),
                                            (128, torch.bfloat16, True), (64, torch.float32, True)],
                         ids=["d128-fp16-causal", "d64-fp16-full", "d128-bf16-causal",
                              "d64-fp32-causal"])
def test_capture_and_replay_equal_eager(d, dtype, causal):
    stage = 3 if dtype == torch.float32 else 5
    if not fused_attn.is_available() or not fused_attn.impl_supports(stage, dtype, d):
        pytest.skip("kernel not available")
    q, k, v = make_qkv(2, 4, 384, d, dtype=dtype, device="cuda", seed=91)
    o_ref, lse_ref = fused_attn.forward(q, k, v, is_causal=causal, return_lse=True)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        fused_attn.forward(q, k, v, is_causal=causal)  # warm-up on the capture stream
        with torch.cuda.graph(g, stream=s):
            o, lse = fused_attn.forward(q, k, v, is_causal=causal, return_lse=True)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        o.zero_()
        lse.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref)
    # new inputs in the captured buffers: the replay computes on them
    q2, k2, v2 = make_qkv(2, 4, 384, d, dtype=dtype, device="cuda", seed=92)
    q.copy_(q2)
    k.copy_(k2)
    v.copy_(v2)
    g.replay()
    torch.cuda.synchronize()
    o2, lse2 = fused_attn.forward(q2, k2, v2, is_causal=causal, return_lse=True)
    assert torch.equal(o, o2) and torch.equal(lse, lse2)
    assert fused_attn.last_device_error() == (0, 0)
    del g
