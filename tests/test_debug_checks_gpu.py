"""The FA_DEBUG_CHECKS build (fused_attn/libfa_sm100_checks.so) against the release build.

The survey's plan for the reference's compute-sanitizer gate (scripts/gpu_run.sh:157-180), which
is closed on this pool: the kernels built with device-side index and address checks (tensor-memory
columns, shared-memory staging offsets, work items, LSE / O indices) that record a status bit and
skip the access instead of trapping.  Over shapes that reach every kernel and path -- both kernels,
fp16 / bf16 / fp32, causal and full, ragged N, GQA, strided views, many items per CTA -- the checked
build must report no failed check (fa_last_device_error == 0) and produce the release build's
output bit for bit.
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

from fused_attn import abi
from fused_attn.workloads import make_qkv

pytestmark = pytest.mark.gpu

CODES = {torch.float16: abi.FA_DTYPE_F16, torch.bfloat16: abi.FA_DTYPE_BF16,
         torch.float32: abi.FA_DTYPE_F32}


@pytest.fixture(scope="module")
def libs():
    if not abi.available() or not abi.CHECKS_LIB_PATH.exists():
        pytest.skip("libfa_sm100.so / libfa_sm100_checks.so not built")
    return abi.lib(), abi.load_checks()


def run(L, q, k, v, causal, block_n=0, strided=None):
    b, h, n, d = q.shape
    dt = CODES[q.dtype]
    impl = abi.FA_IMPL_FUSED if q.dtype == torch.float32 else abi.FA_IMPL_TUNED
    p = abi.params(b, h, k.shape[1], n, d, 1.0 / math.sqrt(d), causal)
    o = torch.full_like(q, float("nan")) if strided is None else strided
    lse = torch.full((b, h, n), float("nan"), device="cuda")
    need = L.fa_workspace_bytes(impl, dt, ctypes.byref(p))
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    L.fa_set_debug_overrides(0, block_n)
    try:
        if strided is None:
            rc = L.fa_forward(impl, dt, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                              lse.data_ptr(), ws.data_ptr(), ctypes.byref(p), stream)
        else:
            st = abi.strides(q, k, v, o)
            rc = L.fa_forward_strided(impl, dt, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                      o.data_ptr(), lse.data_ptr(), ws.data_ptr(), ctypes.byref(p),
                                      ctypes.byref(st), stream)
    finally:
        L.fa_set_debug_overrides(0, 0)
    assert rc == 0
    detail = ctypes.c_uint(0)
    status = L.fa_last_device_error(ctypes.byref(detail))
    return o, lse, status, detail.value


CASES = [
    # (B, H, Hkv, N, D, dtype, causal, block_n)
    (2, 8, 8, 2048, 128, torch.float16, True, 0),     # C3: lookahead kernel
    (2, 8, 8, 2048, 64, torch.float16, False, 0),     # C2: 128-key kernel
    (2, 3, 3, 416, 128, torch.bfloat16, True, 0),     # ragged N, bf16 first-tile P_hi + P_lo
    (2, 3, 3, 160, 64, torch.bfloat16, False, 128),
    (1, 6, 3, 352, 64, torch.float16, True, 64),      # GQA
    (1, 8, 1, 256, 128, torch.bfloat16, False, 32),   # MQA, 32-key tiles
    (16, 48, 48, 160, 64, torch.float16, True, 0),    # many short items per CTA
    (1, 2, 2, 384, 128, torch.float32, True, 0),      # fp32: tf32 pre-pass + 64-key tiles
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[0]}H{c[1]}kv{c[2]}N{c[3]}D{c[4]}-"
                         f"{str(c[5])[6:]}-{'causal' if c[6] else 'full'}-bn{c[7]}")
def test_checked_build_reports_nothing_and_matches_release(libs, case):
    rel, chk = libs
    b, h, hkv, n, d, dt, causal, bn = case
    q, k, v = make_qkv(b, h, n, d, dtype=dt, device="cuda", hkv=hkv, seed=41)
    o_r, l_r, s_r, _ = run(rel, q, k, v, causal, bn)
    o_c, l_c, s_c, bits = run(chk, q, k, v, causal, bn)
    assert s_r == 0
    assert s_c == 0, f"checked build status {s_c} (bits {bits:#x})"
    assert torch.equal(o_c, o_r) and torch.equal(l_c, l_r)


def test_checked_build_on_strided_views(libs):
    rel, chk = libs
    b, t, h, d = 2, 320, 6, 64
    x = torch.randn(b, t, 3, h, d, dtype=torch.float16, device="cuda")
    q, k, v = (x[:, :, i].transpose(1, 2) for i in range(3))  # [B, H, T, D] views
    outs = []
    for L in (rel, chk):
        o = torch.full((b, t, h, d), float("nan"), dtype=torch.float16, device="cuda").transpose(1, 2)
        o, lse, status, bits = run(L, q, k, v, True, 0, strided=o)
        assert status == 0, bits
        outs.append((o, lse))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
