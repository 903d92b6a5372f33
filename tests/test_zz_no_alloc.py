"""fa_forward_noalloc: the forward with scratch from the library's fixed device array.

For callers that cannot allocate device memory when they call (a host function enqueued on a
stream may make no CUDA API calls; some runtimes reserve all device memory up front and give a
plugin no allocator): the fp32 path's 64 MiB of scratch lives in the library, not in a workspace.

Collected last (file name) but independent of the other tests: every case compares the
no-allocation entry point with fa_forward given an explicit workspace, on two calls in a row
(the second call reuses the scratch the first one left behind).
"""

from __future__ import annotations

import math

import pytest
import torch

import fused_attn
from fused_attn import abi
from fused_attn.workloads import make_qkv

pytestmark = pytest.mark.gpu


def require():
    if not fused_attn.is_available():
        pytest.skip("fused_attn._C is not built")
    if not fused_attn.impl_supports(3, torch.float32, 64):
        pytest.skip("fp32 path not built for this device")


def _outputs(q):
    b, h, n, _ = q.shape
    return (torch.full_like(q, float("nan")),
            torch.full((b, h, n), float("nan"), device=q.device, dtype=torch.float32))


@pytest.mark.parametrize("b,h,n,d,causal", [(1, 2, 128, 64, True), (2, 3, 352, 128, False),
                                            (2, 4, 1024, 128, True)])
def test_fp32_two_calls_equal_the_workspace_path(b, h, n, d, causal):
    require()
    p = abi.params(b, h, h, n, d, 1.0 / math.sqrt(d), causal)
    need = abi.workspace_bytes(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, p)
    assert 0 < need <= abi.noalloc_scratch_bytes()
    stream = torch.cuda.current_stream().cuda_stream
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    results = []
    for seed in (81, 82):  # two calls in a row, different inputs
        q, k, v = make_qkv(b, h, n, d, dtype=torch.float32, device="cuda", seed=seed)
        o_ref, lse_ref = _outputs(q)
        o, lse = _outputs(q)
        ptrs = (q.data_ptr(), k.data_ptr(), v.data_ptr())
        assert abi.forward(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, *ptrs, o_ref.data_ptr(),
                           lse_ref.data_ptr(), p, stream, ws.data_ptr()) == 0
        assert abi.forward_noalloc(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, *ptrs, o.data_ptr(),
                                   lse.data_ptr(), p, stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref)
        results.append(o)
    assert not torch.equal(results[0], results[1])
    assert fused_attn.last_device_error() == (0, 0)


def test_fp16_needs_no_scratch():
    require()
    b, h, n, d = 2, 2, 256, 128
    q, k, v = make_qkv(b, h, n, d, dtype=torch.float16, device="cuda", seed=83)
    p = abi.params(b, h, h, n, d, 1.0 / math.sqrt(d), True)
    assert abi.workspace_bytes(abi.FA_IMPL_TUNED, abi.FA_DTYPE_F16, p) == 0
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        o, lse = _outputs(q)
        assert abi.forward_noalloc(abi.FA_IMPL_TUNED, abi.FA_DTYPE_F16, q.data_ptr(), k.data_ptr(),
                                   v.data_ptr(), o.data_ptr(), lse.data_ptr(), p, stream) == 0
        torch.cuda.synchronize()
        o_ref, lse_ref = fused_attn.forward(q, k, v, is_causal=True, return_lse=True)
        assert torch.equal(o, o_ref) and torch.equal(lse, lse_ref)


def test_problem_beyond_the_scratch_is_rejected():
    require()
    # 4 * D * N * (B*H + 2*B*Hkv) bytes: B=8, H=16, N=4096, D=128 needs 768 MiB > 64 MiB.
    p = abi.params(8, 16, 16, 4096, 128, 0.0884, True)
    assert abi.workspace_bytes(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, p) > abi.noalloc_scratch_bytes()
    dummy = torch.empty(16, dtype=torch.float32, device="cuda")
    ptr = dummy.data_ptr()
    assert abi.forward_noalloc(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, ptr, ptr, ptr, ptr, ptr, p) == \
        abi.CUDA_ERROR_INVALID_VALUE
