"""CPU oracle for the SDPA forward -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import this package, and only as the checker or the CPU baseline.
The product path (``fused_attn`` / ``libfa_sm100.so``) never imports it.

Three implementations of the same function, all fp64:

* ``attention`` / ``rows`` / ``tiled``  -- ``oracle/fa_oracle.c``, a C restatement of the
  reference's ``src/reference/cpu_reference.cpp`` (direct softmax :47-92, tiled recurrence
  :94-165), loaded through ctypes from ``oracle/libfa_oracle.so``.
* ``ref_attention`` / ``ref_rows`` / ``ref_tiled`` -- the reference's own
  ``cpu_reference.cpp`` compiled where it lies into ``oracle/_ref/libfa_ref.so``
  (``make -C oracle ref``).  Used to pin the restatement and as the timed CPU baseline.
* ``numpy_attention`` -- a vectorised numpy restatement of the direct form, a third opinion.

Parity is pinned (see tests/test_oracle_cpu.py): the restatement is checked against the
reference's known answers (src/reference/test_cpu_reference.cpp:39-67), its tiled==direct
property, and against fixtures produced by the reference's own oracle and by
``python/fused_attn/reference.py::math_reference`` (tests/golden/gen_golden.py).
"""

from __future__ import annotations

import ctypes
import math
import os
from pathlib import Path
from typing import NamedTuple

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libfa_oracle.so"
REF_LIB_PATH = HERE / "_ref" / "libfa_ref.so"
LOG2E = 1.4426950408889634

_c_double_p = ctypes.POINTER(ctypes.c_double)


class _Shape(ctypes.Structure):
    _fields_ = [
        ("B", ctypes.c_int),
        ("H", ctypes.c_int),
        ("Hkv", ctypes.c_int),
        ("N", ctypes.c_int),
        ("D", ctypes.c_int),
        ("scale", ctypes.c_double),
        ("causal", ctypes.c_int),
    ]


_lib = None
_ref = None


def reference_root() -> Path:
    """The reference checkout: $FA_REFERENCE_ROOT, else a `reference` directory beside this
    repository (it need not exist: the reference-compiled oracle is then simply not built)."""
    env = os.environ.get("FA_REFERENCE_ROOT")
    return Path(env) if env else HERE.parent.parent / "reference"


def build(ref: bool | None = None, quiet: bool = True) -> None:
    """Compile ``libfa_oracle.so`` (and ``_ref`` when the reference tree is present)."""
    import subprocess

    targets = ["all"]
    ref_root = reference_root()
    if ref is None:
        ref = (ref_root / "src" / "reference" / "cpu_reference.cpp").exists()
    if ref:
        targets.append("ref")
    subprocess.run(
        ["make", "-C", str(HERE), f"REF={ref_root}", *targets],
        check=True,
        stdout=subprocess.DEVNULL if quiet else None,
    )


def _load():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build(ref=False)
        lib = ctypes.CDLL(str(LIB_PATH))
        sp = ctypes.POINTER(_Shape)
        lib.fa_oracle_attention.argtypes = [_c_double_p] * 3 + [sp, _c_double_p, _c_double_p, ctypes.c_int]
        lib.fa_oracle_attention.restype = ctypes.c_int
        lib.fa_oracle_rows.argtypes = [_c_double_p] * 3 + [sp] + [ctypes.c_int] * 4 + [_c_double_p] * 2
        lib.fa_oracle_rows.restype = None
        lib.fa_oracle_tiled.argtypes = [_c_double_p] * 3 + [sp] + [ctypes.c_int] * 3 + [_c_double_p] * 2
        lib.fa_oracle_tiled.restype = None
        lib.fa_oracle_max_abs.argtypes = [_c_double_p, _c_double_p, ctypes.c_size_t]
        lib.fa_oracle_max_abs.restype = ctypes.c_double
        _lib = lib
    return _lib


def ref_available() -> bool:
    return REF_LIB_PATH.exists()


def _load_ref():
    global _ref
    if _ref is None:
        if not REF_LIB_PATH.exists():
            raise FileNotFoundError(
                f"{REF_LIB_PATH} is not built (make -C oracle ref with the reference tree present)"
            )
        lib = ctypes.CDLL(str(REF_LIB_PATH))
        i, d = ctypes.c_int, ctypes.c_double
        lib.fa_ref_attention.argtypes = [_c_double_p] * 3 + [i] * 5 + [d, i, _c_double_p, _c_double_p, i]
        lib.fa_ref_attention.restype = ctypes.c_int
        lib.fa_ref_rows.argtypes = [_c_double_p] * 3 + [i] * 5 + [d, i] + [i] * 4 + [_c_double_p] * 2
        lib.fa_ref_rows.restype = None
        lib.fa_ref_attention_tiled.argtypes = (
            [_c_double_p] * 3 + [i] * 5 + [d, i, i, i, _c_double_p, _c_double_p]
        )
        lib.fa_ref_attention_tiled.restype = None
        _ref = lib
    return _ref


# ---------------------------------------------------------------------------------------------
def _as_f64(x) -> np.ndarray:
    """Upcast any float array (numpy, or a torch tensor of any device/dtype) to C-contiguous f64.

    fp16/bf16 values are exactly representable in fp64, so the oracle sees the very values the
    kernel saw (the reference's self-check does the same, bench/bench_main.cu:632-640)."""
    if hasattr(x, "detach"):  # torch tensor
        x = x.detach().to("cpu").double().numpy()
    return np.ascontiguousarray(np.asarray(x, dtype=np.float64))


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_c_double_p)


def _shape(q: np.ndarray, k: np.ndarray, scale: float | None, causal: bool) -> _Shape:
    if q.ndim != 4 or k.ndim != 4:
        raise ValueError("q, k, v must be [B, H, N, D]")
    b, h, n, d = q.shape
    hkv = k.shape[1]
    if h % hkv:
        raise ValueError(f"H={h} must be a multiple of Hkv={hkv}")
    if k.shape[2] != n:
        raise ValueError("Nq == Nkv is required")
    sc = 1.0 / math.sqrt(d) if scale is None else float(scale)
    return _Shape(b, h, hkv, n, d, sc, 1 if causal else 0)


def default_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def attention(q, k, v, causal: bool = False, scale: float | None = None, threads: int = 1):
    """fp64 (o, lse) for the whole tensor: the C restatement, on ``threads`` threads."""
    q64, k64, v64 = _as_f64(q), _as_f64(k), _as_f64(v)
    s = _shape(q64, k64, scale, causal)
    o = np.empty_like(q64)
    lse = np.empty(q64.shape[:3], dtype=np.float64)
    _load().fa_oracle_attention(_ptr(q64), _ptr(k64), _ptr(v64), ctypes.byref(s), _ptr(o), _ptr(lse), int(threads))
    return o, lse


def rows(q, k, v, b: int, h: int, row0: int, nrows: int, causal: bool = False, scale: float | None = None):
    """fp64 (o, lse) for rows [row0, row0 + nrows) of head (b, h)."""
    q64, k64, v64 = _as_f64(q), _as_f64(k), _as_f64(v)
    s = _shape(q64, k64, scale, causal)
    o = np.empty((nrows, q64.shape[3]), dtype=np.float64)
    lse = np.empty((nrows,), dtype=np.float64)
    _load().fa_oracle_rows(_ptr(q64), _ptr(k64), _ptr(v64), ctypes.byref(s), b, h, row0, nrows, _ptr(o), _ptr(lse))
    return o, lse


def tiled(q, k, v, block_m: int, block_n: int, causal: bool = False, scale: float | None = None,
          skip_masked: bool = True):
    """fp64 (o, lse) through the tiled online-softmax recurrence (the kernels' algorithm)."""
    if block_m <= 0 or block_n <= 0:
        raise ValueError("block_m and block_n must be positive")
    q64, k64, v64 = _as_f64(q), _as_f64(k), _as_f64(v)
    s = _shape(q64, k64, scale, causal)
    o = np.empty_like(q64)
    lse = np.empty(q64.shape[:3], dtype=np.float64)
    _load().fa_oracle_tiled(_ptr(q64), _ptr(k64), _ptr(v64), ctypes.byref(s), int(block_m), int(block_n),
                            1 if skip_masked else 0, _ptr(o), _ptr(lse))
    return o, lse


def ref_attention(q, k, v, causal: bool = False, scale: float | None = None, threads: int = 1):
    """The reference's own fa::ref::attention_rows, threaded over heads (oracle/_ref)."""
    q64, k64, v64 = _as_f64(q), _as_f64(k), _as_f64(v)
    s = _shape(q64, k64, scale, causal)
    o = np.empty_like(q64)
    lse = np.empty(q64.shape[:3], dtype=np.float64)
    used = _load_ref().fa_ref_attention(_ptr(q64), _ptr(k64), _ptr(v64), s.B, s.H, s.Hkv, s.N, s.D,
                                        s.scale, s.causal, _ptr(o), _ptr(lse), int(threads))
    return o, lse, used


def ref_rows(q, k, v, b: int, h: int, row0: int, nrows: int, causal: bool = False, scale: float | None = None):
    q64, k64, v64 = _as_f64(q), _as_f64(k), _as_f64(v)
    s = _shape(q64, k64, scale, causal)
    o = np.empty((nrows, q64.shape[3]), dtype=np.float64)
    lse = np.empty((nrows,), dtype=np.float64)
    _load_ref().fa_ref_rows(_ptr(q64), _ptr(k64), _ptr(v64), s.B, s.H, s.Hkv, s.N, s.D, s.scale,
                            s.causal, b, h, row0, nrows, _ptr(o), _ptr(lse))
    return o, lse


def ref_tiled(q, k, v, block_m: int, block_n: int, causal: bool = False, scale: float | None = None):
    q64, k64, v64 = _as_f64(q), _as_f64(k), _as_f64(v)
    s = _shape(q64, k64, scale, causal)
    o = np.empty_like(q64)
    lse = np.empty(q64.shape[:3], dtype=np.float64)
    _load_ref().fa_ref_attention_tiled(_ptr(q64), _ptr(k64), _ptr(v64), s.B, s.H, s.Hkv, s.N, s.D,
                                       s.scale, s.causal, int(block_m), int(block_n), _ptr(o), _ptr(lse))
    return o, lse


def numpy_attention(q, k, v, causal: bool = False, scale: float | None = None, keep=None):
    """Vectorised fp64 direct softmax (small shapes).  ``keep`` is an optional boolean
    [N, N] "attend" mask, used only to drive the fully-masked-row guards in the tests."""
    q64, k64, v64 = _as_f64(q), _as_f64(k), _as_f64(v)
    b, h, n, d = q64.shape
    rep = h // k64.shape[1]
    if rep != 1:
        k64 = np.repeat(k64, rep, axis=1)
        v64 = np.repeat(v64, rep, axis=1)
    sc = 1.0 / math.sqrt(d) if scale is None else float(scale)
    s = np.einsum("bhid,bhjd->bhij", q64, k64) * sc
    mask = np.ones((n, n), dtype=bool)
    if causal:
        mask &= np.tril(np.ones((n, n), dtype=bool))
    if keep is not None:
        mask &= np.asarray(keep, dtype=bool)
    s = np.where(mask, s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    m_safe = np.where(np.isneginf(m), 0.0, m)
    p = np.exp(s - m_safe)
    l = p.sum(axis=-1, keepdims=True)
    inv = np.where(l == 0, 0.0, 1.0 / np.where(l == 0, 1.0, l))
    o = np.einsum("bhij,bhjd->bhid", p, v64) * inv
    with np.errstate(divide="ignore"):
        lse = np.where(l == 0, np.inf, m_safe + np.log(np.where(l == 0, 1.0, l)))
    return o, lse[..., 0]


def combine(o_parts, lse_parts):
    """LSE-weighted merge of attention partials over disjoint key sets, fp64:
    lse = ln sum_i exp(lse_i), o = sum_i exp(lse_i - lse) o_i.  A partial row with lse = +inf
    (the forward's "saw no key" value, cpu_reference.cpp / softmax_math.cuh:64-68) or -inf has
    weight 0; a row with no keys anywhere gives o = 0, lse = +inf.  The reference has no combine
    of its own (its roadmap lists one); this restates the math it implies, and the CPU tests pin
    it to ``numpy_attention`` on the unsplit keys."""
    lse = np.stack([_as_f64(x) for x in lse_parts])  # [S, B, H, N]
    o = np.stack([_as_f64(x) for x in o_parts])      # [S, B, H, N, D]
    empty = ~np.isfinite(lse)
    m = np.where(empty, -np.inf, lse).max(axis=0)
    has = np.isfinite(m)
    m_safe = np.where(has, m, 0.0)
    w = np.where(empty, 0.0, np.exp(np.where(empty, 0.0, lse) - m_safe))
    l = w.sum(axis=0)
    ok = l > 0
    out = (w[..., None] * o).sum(axis=0) / np.where(ok, l, 1.0)[..., None]
    out = np.where(ok[..., None], out, 0.0)
    lse_out = np.where(ok, m_safe + np.log(np.where(ok, l, 1.0)), np.inf)
    return out, lse_out


def max_abs(a, b) -> float:
    """NaN-aware max |a - b| (cpu_reference.cpp:167-175): NaN anywhere counts as +inf."""
    a64, b64 = _as_f64(a), _as_f64(b)
    d = np.abs(a64 - b64)
    if np.isnan(d).any():
        return math.inf
    return float(d.max()) if d.size else 0.0


# ---------------------------------------------------------------------------------------------
class RatioResult(NamedTuple):
    """FlashAttention ratio rule outcome (python/fused_attn/reference.py:314-352)."""

    err_mine: float
    err_torch: float
    bound: float
    ok: bool
    out_finite: bool
    torch_finite: bool


def error_ratio(out, ref64, same_dtype) -> RatioResult:
    """``err_mine <= 2 * err_same_dtype + 1e-6``: the reference's secondary gate
    (reference.py:331-352).  ``same_dtype`` is a naive attention computed in the input dtype."""
    o = _as_f64(out)
    r = _as_f64(ref64)
    t = _as_f64(same_dtype)
    err_mine = float(np.abs(o - r).max())
    err_torch = float(np.abs(t - r).max())
    bound = 2.0 * err_torch + 1e-6
    out_finite = bool(np.isfinite(o).all())
    torch_finite = math.isfinite(err_torch)
    ok = out_finite and torch_finite and err_mine <= bound
    return RatioResult(err_mine, err_torch, bound, ok, out_finite, torch_finite)

