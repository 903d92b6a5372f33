"""ctypes binding of the C ABI in include/fa_sm100.h (``libfa_sm100.so``).

This is the FFI a non-torch host (the reference's torch-free ``fa_bench``, or any cgo / JNI /
N-API caller) would use; the tests drive the kernel through it directly, and the torch
extension (``fused_attn._C``) links the same library, so both paths share one process-global
state (debug overrides, wait-time limit, device status word).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfa_sm100.so"
CHECKS_LIB_PATH = Path(__file__).resolve().parent / "libfa_sm100_checks.so"

# Every function declared in include/fa_sm100.h (the CPU test checks the header and this list
# against the library's exported symbols).
EXPORTS = (
    "fa_forward",
    "fa_forward_strided",
    "fa_combine",
    "fa_forward_noalloc",
    "fa_noalloc_scratch_bytes",
    "fa_workspace_bytes",
    "fa_impl_supports",
    "fa_set_debug_overrides",
    "fa_get_debug_overrides",
    "fa_impl_name",
    "fa_dtype_name",
    "fa_dtype_size",
    "fa_last_device_error",
    "fa_set_wait_timeout_ns",
    "fa_debug_set_skip_kv_tile",
)

FA_DTYPE_F32, FA_DTYPE_F16, FA_DTYPE_BF16 = 0, 1, 2
FA_IMPL_NAIVE, FA_IMPL_TILED, FA_IMPL_FUSED, FA_IMPL_WMMA, FA_IMPL_TUNED = 1, 2, 3, 4, 5

CUDA_SUCCESS = 0
CUDA_ERROR_INVALID_VALUE = 1
CUDA_ERROR_LAUNCH_TIMEOUT = 702
CUDA_ERROR_NOT_SUPPORTED = 801


class FaParams(ctypes.Structure):
    """``fa_params_t`` (fa::Params, attention.cuh:28-36)."""

    _fields_ = [
        ("B", ctypes.c_int),
        ("H", ctypes.c_int),
        ("Hkv", ctypes.c_int),
        ("N", ctypes.c_int),
        ("D", ctypes.c_int),
        ("scale", ctypes.c_float),
        ("causal", ctypes.c_int),
    ]


class FaStrides(ctypes.Structure):
    """``fa_strides_t``: element strides of the (b, h, n) dims of q, k, v, o (d contiguous)."""

    _fields_ = [("q", ctypes.c_longlong * 3), ("k", ctypes.c_longlong * 3),
                ("v", ctypes.c_longlong * 3), ("o", ctypes.c_longlong * 3)]


_lib: ctypes.CDLL | None = None


def available() -> bool:
    return LIB_PATH.exists()


def lib() -> ctypes.CDLL:
    """Load ``libfa_sm100.so`` (raises if it was not built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is not built; run `python fused-attention-cuda_b200/build.py`"
            )
        _lib = configure(ctypes.CDLL(str(LIB_PATH)))
    return _lib


def configure(L: ctypes.CDLL) -> ctypes.CDLL:
    """Sets the argument and result types of every exported function on a loaded library (the
    release libfa_sm100.so or its FA_DEBUG_CHECKS build)."""
    vp, i, u = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint
    L.fa_forward.argtypes = [i, i, vp, vp, vp, vp, vp, vp, ctypes.POINTER(FaParams), vp]
    L.fa_forward.restype = i
    L.fa_forward_strided.argtypes = [i, i, vp, vp, vp, vp, vp, vp, ctypes.POINTER(FaParams),
                                     ctypes.POINTER(FaStrides), vp]
    L.fa_forward_strided.restype = i
    L.fa_combine.argtypes = [i, i, ctypes.POINTER(vp), ctypes.POINTER(vp), vp, vp, i, i, i, i,
                             vp]
    L.fa_combine.restype = i
    L.fa_forward_noalloc.argtypes = [i, i, vp, vp, vp, vp, vp, ctypes.POINTER(FaParams), vp]
    L.fa_forward_noalloc.restype = i
    L.fa_noalloc_scratch_bytes.argtypes = []
    L.fa_noalloc_scratch_bytes.restype = ctypes.c_size_t
    L.fa_workspace_bytes.argtypes = [i, i, ctypes.POINTER(FaParams)]
    L.fa_workspace_bytes.restype = ctypes.c_size_t
    L.fa_impl_supports.argtypes = [i, i, i, i]
    L.fa_impl_supports.restype = i
    L.fa_set_debug_overrides.argtypes = [i, i]
    L.fa_set_debug_overrides.restype = None
    L.fa_get_debug_overrides.argtypes = [i, ctypes.POINTER(i), ctypes.POINTER(i)]
    L.fa_get_debug_overrides.restype = None
    L.fa_impl_name.argtypes = [i]
    L.fa_impl_name.restype = ctypes.c_char_p
    L.fa_dtype_name.argtypes = [i]
    L.fa_dtype_name.restype = ctypes.c_char_p
    L.fa_dtype_size.argtypes = [i]
    L.fa_dtype_size.restype = ctypes.c_size_t
    L.fa_last_device_error.argtypes = [ctypes.POINTER(u)]
    L.fa_last_device_error.restype = i
    L.fa_set_wait_timeout_ns.argtypes = [ctypes.c_ulonglong]
    L.fa_set_wait_timeout_ns.restype = None
    L.fa_debug_set_skip_kv_tile.argtypes = [i]
    L.fa_debug_set_skip_kv_tile.restype = None
    return L


def load_checks() -> ctypes.CDLL:
    """The FA_DEBUG_CHECKS build (libfa_sm100_checks.so: device index checks that report
    cudaErrorAssert instead of trapping), a separate library instance with its own state."""
    if not CHECKS_LIB_PATH.exists():
        raise ImportError(f"{CHECKS_LIB_PATH} is not built")
    return configure(ctypes.CDLL(str(CHECKS_LIB_PATH)))


def params(B: int, H: int, Hkv: int, N: int, D: int, scale: float, causal: bool) -> FaParams:
    return FaParams(int(B), int(H), int(Hkv), int(N), int(D), float(scale), 1 if causal else 0)


def forward(impl: int, dtype: int, q: int, k: int, v: int, o: int, lse: int, p: FaParams,
            stream: int = 0, workspace: int = 0) -> int:
    """Raw ``fa_forward`` on device pointers (ints); returns the cudaError_t value."""
    return int(lib().fa_forward(impl, dtype, q, k, v, o, lse, workspace or None,
                                ctypes.byref(p), stream or None))


def strides(q, k, v, o) -> FaStrides:
    """FaStrides of four [B, H, N, D] tensors (anything with ``.stride()``)."""
    st = FaStrides()
    for name, t in (("q", q), ("k", k), ("v", v), ("o", o)):
        sb, sh, sn, _ = t.stride()
        getattr(st, name)[:] = [int(sb), int(sh), int(sn)]
    return st


def forward_strided(impl: int, dtype: int, q: int, k: int, v: int, o: int, lse: int,
                    p: FaParams, st: FaStrides | None, stream: int = 0, workspace: int = 0) -> int:
    """Raw ``fa_forward_strided``; ``st=None`` passes NULL (an invalid-value error)."""
    return int(lib().fa_forward_strided(impl, dtype, q, k, v, o, lse, workspace or None,
                                        ctypes.byref(p), ctypes.byref(st) if st is not None else None,
                                        stream or None))


def forward_noalloc(impl: int, dtype: int, q: int, k: int, v: int, o: int, lse: int,
                    p: FaParams, stream: int = 0) -> int:
    """Raw ``fa_forward_noalloc`` (scratch from the library's fixed device array)."""
    return int(lib().fa_forward_noalloc(impl, dtype, q, k, v, o, lse, ctypes.byref(p),
                                        stream or None))


def noalloc_scratch_bytes() -> int:
    return int(lib().fa_noalloc_scratch_bytes())


COMBINE_MAX_SPLITS = 64


def combine(dtype: int, o_parts: list[int], lse_parts: list[int], o: int, lse: int, B: int,
            H: int, N: int, D: int, stream: int = 0) -> int:
    """Raw ``fa_combine`` on device pointers; returns the cudaError_t value."""
    n = len(o_parts)
    op = (ctypes.c_void_p * max(n, 1))(*o_parts)
    lp = (ctypes.c_void_p * max(n, 1))(*lse_parts)
    return int(lib().fa_combine(dtype, n, op, lp, o, lse, B, H, N, D, stream or None))


def impl_supports(impl: int, dtype: int, D: int, sm: int) -> bool:
    return bool(lib().fa_impl_supports(impl, dtype, D, sm))


def impl_name(impl: int) -> str:
    return lib().fa_impl_name(impl).decode()


def dtype_name(dtype: int) -> str:
    return lib().fa_dtype_name(dtype).decode()


def dtype_size(dtype: int) -> int:
    return int(lib().fa_dtype_size(dtype))


def workspace_bytes(impl: int, dtype: int, p: FaParams) -> int:
    return int(lib().fa_workspace_bytes(impl, dtype, ctypes.byref(p)))


def set_debug_overrides(block_m: int = 0, block_n: int = 0) -> None:
    lib().fa_set_debug_overrides(int(block_m), int(block_n))


def get_debug_overrides(from_env: bool = True) -> tuple[int, int]:
    bm, bn = ctypes.c_int(0), ctypes.c_int(0)
    lib().fa_get_debug_overrides(1 if from_env else 0, ctypes.byref(bm), ctypes.byref(bn))
    return bm.value, bn.value


def last_device_error() -> tuple[int, int]:
    """(cudaError_t, cause bits) of the bounded device waits since the previous call.
    Synchronises the current device."""
    bits = ctypes.c_uint(0)
    err = int(lib().fa_last_device_error(ctypes.byref(bits)))
    return err, int(bits.value)


def set_wait_timeout_ns(ns: int) -> None:
    lib().fa_set_wait_timeout_ns(int(ns))


def debug_set_skip_kv_tile(tile: int) -> None:
    lib().fa_debug_set_skip_kv_tile(int(tile))


DTYPE_CODES = {"fp32": FA_DTYPE_F32, "fp16": FA_DTYPE_F16, "bf16": FA_DTYPE_BF16}


def dtype_code(torch_dtype) -> int:
    import torch

    return {torch.float32: FA_DTYPE_F32, torch.float16: FA_DTYPE_F16,
            torch.bfloat16: FA_DTYPE_BF16}[torch_dtype]
