"""fa_forward_noalloc: the forward with scratch from the library's fixed device array.

For callers that cannot allocate device memory when they call (a plugin in a runtime that reserves
all device memory up front and hands it no allocator): the fp32 path's 64 MiB of scratch lives in
the library, not in a workspace.

Collected last (file name) and independent of the other tests: every case compares the
no-allocation entry point with fa_forward given an explicit workspace, on two calls in a row (the
second call reuses the scratch the first one left behind).  Further cases check that calls after
the first leave free device memory unchanged, and that a call made in a second CUDA context (one
a plugin could have created with the driver API) uses that context's array.
"""

from __future__ import annotations

import math
import subprocess
import sys

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


def test_calls_after_the_first_allocate_no_device_memory():
    require()
    b, h, n, d = 2, 4, 512, 128
    p = abi.params(b, h, h, n, d, 1.0 / math.sqrt(d), True)
    stream = torch.cuda.current_stream().cuda_stream
    inputs = [make_qkv(b, h, n, d, dtype=torch.float32, device="cuda", seed=s) for s in (84, 85)]
    o, lse = _outputs(inputs[0][0])

    def call(q, k, v):
        return abi.forward_noalloc(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, q.data_ptr(), k.data_ptr(),
                                   v.data_ptr(), o.data_ptr(), lse.data_ptr(), p, stream)

    assert call(*inputs[0]) == 0  # the first call may load the module (and the array with it)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    used0 = torch.cuda.memory_allocated()
    for q, k, v in inputs:
        assert call(q, k, v) == 0
        torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.cuda.memory_allocated() == used0
    assert fused_attn.last_device_error() == (0, 0)


# Runs in a fresh process with no torch: the primary context first, then a context created with
# the driver API (as a plugin might), each with its own buffers; in both, fa_forward_noalloc must
# equal fa_forward with an explicit workspace, bit for bit.
_SECOND_CONTEXT = r"""
import ctypes, importlib.util, math, sys
import numpy as np
from cuda.bindings import driver as cu

spec = importlib.util.spec_from_file_location("fa_abi", sys.argv[1])
abi = importlib.util.module_from_spec(spec)
spec.loader.exec_module(abi)

def ok(r):
    err = r[0] if isinstance(r, tuple) else r
    if err != cu.CUresult.CUDA_SUCCESS:
        raise SystemExit(f"driver call failed: {err}")
    return r[1] if isinstance(r, tuple) and len(r) > 1 else None

def run_in_current_context(tag, seed):
    b, h, n, d = 1, 2, 256, 64
    p = abi.params(b, h, h, n, d, 1.0 / math.sqrt(d), True)
    rng = np.random.default_rng(seed)
    host = [rng.standard_normal((b, h, n, d), dtype=np.float32) for _ in range(3)]
    nbytes = host[0].nbytes
    need = int(abi.lib().fa_workspace_bytes(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, ctypes.byref(p)))
    bufs = []
    def alloc(size):
        ptr = int(ok(cu.cuMemAlloc(size)))
        bufs.append(ptr)
        return ptr
    q, k, v = (alloc(nbytes) for _ in range(3))
    for ptr, arr in zip((q, k, v), host):
        ok(cu.cuMemcpyHtoD(ptr, arr.ctypes.data, nbytes))
    ws = alloc(need)
    outs = [(alloc(nbytes), alloc(b * h * n * 4)) for _ in range(3)]
    assert abi.forward(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, q, k, v, outs[0][0], outs[0][1], p,
                       0, ws) == 0
    for o, lse in outs[1:]:  # two calls in a row
        rc = abi.forward_noalloc(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, q, k, v, o, lse, p, 0)
        if rc != 0:
            raise SystemExit(f"{tag}: fa_forward_noalloc returned {rc}")
    ok(cu.cuCtxSynchronize())
    got = []
    for o, lse in outs:
        ho = np.empty((b, h, n, d), np.float32)
        hl = np.empty((b, h, n), np.float32)
        ok(cu.cuMemcpyDtoH(ho.ctypes.data, o, ho.nbytes))
        ok(cu.cuMemcpyDtoH(hl.ctypes.data, lse, hl.nbytes))
        got.append((ho, hl))
    for ptr in bufs:
        ok(cu.cuMemFree(ptr))
    detail = ctypes.c_uint(0)
    status = abi.lib().fa_last_device_error(ctypes.byref(detail))
    if status != 0:
        raise SystemExit(f"{tag}: device status {status} ({detail.value:#x})")
    ref_o, ref_l = got[0]
    if not np.isfinite(ref_o).all():
        raise SystemExit(f"{tag}: workspace path produced non-finite output")
    for o_, l_ in got[1:]:
        if not (np.array_equal(o_, ref_o) and np.array_equal(l_, ref_l)):
            raise SystemExit(f"{tag}: noalloc output differs from the workspace path")
    print(tag, "ok")

ok(cu.cuInit(0))
dev = ok(cu.cuDeviceGet(0))
primary = ok(cu.cuDevicePrimaryCtxRetain(dev))
ok(cu.cuCtxPushCurrent(primary))
run_in_current_context("primary", 86)
ok(cu.cuCtxPopCurrent())
ctx = ok(cu.cuCtxCreate(0, dev))  # created current
run_in_current_context("second", 87)
ok(cu.cuCtxDestroy(ctx))
ok(cu.cuDevicePrimaryCtxRelease(dev))
"""


def test_second_context_uses_its_own_array():
    require()
    pytest.importorskip("cuda.bindings.driver")
    r = subprocess.run([sys.executable, "-c", _SECOND_CONTEXT, str(abi.LIB_PATH.parent / "abi.py")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "primary ok" in r.stdout and "second ok" in r.stdout
