"""CPU checks of the drop-in boundary (no device work: nothing here launches a kernel).

* libfa_sm100.so loads and exports exactly the functions include/fa_sm100.h declares;
* the scalar helpers (names, sizes, impl_supports, workspace, overrides) behave like the
  reference's (src/dispatch.cu:163-230);
* invalid parameters are rejected with cudaErrorInvalidValue before any CUDA call, as
  fa::forward's validate() does (src/dispatch.cu:96-111).
"""

from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT
from fused_attn import abi

HEADER = ROOT / "include" / "fa_sm100.h"

pytestmark = pytest.mark.skipif(not abi.available(), reason="libfa_sm100.so not built")


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(fa_[a-z_0-9]+)\s*\(", text))


def exported_functions(path=None) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(path or abi.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_library_exports_every_declared_symbol():
    declared = declared_functions()
    assert declared, "no declarations parsed from the header"
    exported = {s for s in exported_functions() if s.startswith("fa_")}
    assert declared <= exported, f"declared but not exported: {declared - exported}"
    assert set(abi.EXPORTS) == declared, "fused_attn.abi.EXPORTS is out of sync with the header"
    lib = abi.lib()
    for name in declared:
        assert hasattr(lib, name)


def test_checks_build_exports_the_same_symbols():
    """libfa_sm100_checks.so (-DFA_DEBUG_CHECKS) is the same C ABI with device index checks."""
    if not abi.CHECKS_LIB_PATH.exists():
        pytest.skip("libfa_sm100_checks.so not built")
    declared = declared_functions()
    exported = {s for s in exported_functions(abi.CHECKS_LIB_PATH) if s.startswith("fa_")}
    assert declared <= exported
    chk = abi.load_checks()
    assert chk.fa_impl_name(5) == b"tuned" and chk.fa_dtype_size(1) == 2


def test_names_and_sizes_match_reference():
    assert [abi.impl_name(i) for i in range(1, 6)] == ["naive", "tiled", "fused", "wmma", "tuned"]
    assert abi.impl_name(0) == "unknown" and abi.impl_name(9) == "unknown"
    assert [abi.dtype_name(i) for i in range(3)] == ["fp32", "fp16", "bf16"]
    assert [abi.dtype_size(i) for i in range(3)] == [4, 2, 2]
    assert abi.dtype_size(7) == 0 and abi.dtype_name(7) == "unknown"


def test_impl_supports_matrix_on_sm100():
    """Stage support as in the reference's contract gate (src/dispatch.cu:76-89), sm_100 only:
    Tuned takes fp16/bf16, Fused takes fp32 (tf32 tensor cores) and fp16; stages 1, 2, 4 are
    not built."""
    want = {
        abi.FA_IMPL_TUNED: {abi.FA_DTYPE_F16, abi.FA_DTYPE_BF16},
        abi.FA_IMPL_FUSED: {abi.FA_DTYPE_F32, abi.FA_DTYPE_F16},
    }
    for dt in (abi.FA_DTYPE_F32, abi.FA_DTYPE_F16, abi.FA_DTYPE_BF16):
        for d in (64, 128):
            for impl in (1, 2, 3, 4, 5):
                ok = dt in want.get(impl, set())
                assert bool(abi.impl_supports(impl, dt, d, 100)) == ok, (impl, dt, d)
                assert not abi.impl_supports(impl, dt, d, 90)
                assert not abi.impl_supports(impl, dt, d, 103)
            assert not abi.impl_supports(abi.FA_IMPL_TUNED, dt, 96, 100)
            assert not abi.impl_supports(abi.FA_IMPL_FUSED, dt, 96, 100)


def test_workspace_bytes():
    """0 for fp16/bf16 (fused kernel, as the reference's fused stages); fp32 on Impl::Fused
    stages tf32-rounded q, k, v: 4*D*N*(B*H + 2*B*Hkv) bytes."""
    p = abi.params(2, 8, 8, 2048, 128, 0.088, True)
    assert abi.workspace_bytes(abi.FA_IMPL_TUNED, abi.FA_DTYPE_F16, p) == 0
    assert abi.workspace_bytes(abi.FA_IMPL_TUNED, abi.FA_DTYPE_BF16, p) == 0
    assert abi.workspace_bytes(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F16, p) == 0
    assert abi.workspace_bytes(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, p) == 4 * 128 * 2048 * (16 + 32)
    g = abi.params(2, 8, 2, 256, 64, 0.125, False)
    assert abi.workspace_bytes(abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, g) == 4 * 64 * 256 * (16 + 8)


def test_debug_overrides_roundtrip_and_env(monkeypatch):
    abi.set_debug_overrides(128, 64)
    assert abi.get_debug_overrides(from_env=False) == (128, 64)
    monkeypatch.setenv("FA_FORCE_BC", "32")
    assert abi.get_debug_overrides(from_env=True) == (128, 32)
    abi.set_debug_overrides(0, 0)
    assert abi.get_debug_overrides(from_env=False) == (0, 0)


P16 = 0x1000  # a 16-byte aligned fake address: validation rejects before it is ever used


@pytest.mark.parametrize(
    "mutate",
    [
        dict(N=100),  # N % 32
        dict(D=96),  # D not in {64, 128}
        dict(Hkv=3),  # H % Hkv
        dict(B=0),
        dict(scale=0.0),
        dict(scale=float("inf")),
        dict(scale=float("nan")),
    ],
    ids=lambda m: ",".join(f"{k}={v}" for k, v in m.items()),
)
def test_invalid_params_rejected_without_device(mutate):
    args = dict(B=1, H=4, Hkv=4, N=128, D=64, scale=0.125, causal=False)
    args.update(mutate)
    p = abi.params(**args)
    err = abi.forward(abi.FA_IMPL_TUNED, abi.FA_DTYPE_F16, P16, P16, P16, P16, P16, p)
    assert err == abi.CUDA_ERROR_INVALID_VALUE


def test_null_and_misaligned_pointers_rejected():
    p = abi.params(1, 2, 2, 128, 64, 0.125, True)
    F16, T = abi.FA_DTYPE_F16, abi.FA_IMPL_TUNED
    assert abi.forward(T, F16, 0, P16, P16, P16, P16, p) == abi.CUDA_ERROR_INVALID_VALUE
    assert abi.forward(T, F16, P16, P16, P16, P16, 0, p) == abi.CUDA_ERROR_INVALID_VALUE  # lse
    assert abi.forward(T, F16, P16 + 8, P16, P16, P16, P16, p) == abi.CUDA_ERROR_INVALID_VALUE
    assert abi.forward(T, 9, P16, P16, P16, P16, P16, p) == abi.CUDA_ERROR_INVALID_VALUE


def test_null_params_pointer_rejected():
    err = abi.lib().fa_forward(5, 1, P16, P16, P16, P16, P16, None, None, None)
    assert err == abi.CUDA_ERROR_INVALID_VALUE


@pytest.mark.parametrize("case", ["null_params", "d96", "n_ragged", "h_not_multiple", "scale0",
                                  "misaligned", "null_lse"])
def test_noalloc_rejects_what_forward_rejects(case):
    """fa_forward_noalloc makes fa_forward's argument checks, with its codes, before it looks up
    its scratch array (fp32 on the fused implementation, the only path that uses it)."""
    good = abi.params(1, 2, 2, 128, 64, 0.125, True)
    ptr, lse = 256, 512
    p = good
    q = ptr
    if case == "d96":
        p = abi.params(1, 2, 2, 128, 96, 0.125, True)
    elif case == "n_ragged":
        p = abi.params(1, 2, 2, 100, 64, 0.125, True)
    elif case == "h_not_multiple":
        p = abi.params(1, 3, 2, 128, 64, 0.125, True)
    elif case == "scale0":
        p = abi.params(1, 2, 2, 128, 64, 0.0, True)
    elif case == "misaligned":
        q = ptr + 4
    elif case == "null_lse":
        lse = 0
    L = abi.lib()
    args = (abi.FA_IMPL_FUSED, abi.FA_DTYPE_F32, q, ptr, ptr, ptr, lse or None)
    pp = None if case == "null_params" else ctypes.byref(p)
    rc_noalloc = L.fa_forward_noalloc(*args, pp, None)
    rc_forward = L.fa_forward(*args, None, pp, None)
    assert rc_noalloc == rc_forward == abi.CUDA_ERROR_INVALID_VALUE
