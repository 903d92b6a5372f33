"""fused_attn -- B200 (sm_100a) fused scaled-dot-product-attention forward for PyTorch.

Drop-in for the reference's ``python/fused_attn`` package: same op library name, same wrapper
functions, same validation messages.  The ops (registered by ``fused_attn._C``)::

    torch.ops.fused_attn.forward(q, k, v, is_causal, scale) -> (O, LSE)
    torch.ops.fused_attn.forward_stage(q, k, v, is_causal, scale, stage) -> (O, LSE)
    torch.ops.fused_attn.forward_strided(q, k, v, is_causal, scale) -> (O, LSE)   [B200 addition]
    torch.ops.fused_attn.combine(o_parts, lse_parts) -> (O, LSE)                 [B200 addition]
    torch.ops.fused_attn.set_debug_overrides(block_m, block_n) -> ()
    torch.ops.fused_attn.impl_supports(stage, dtype_name, D) -> bool
    torch.ops.fused_attn.impl_name(stage) -> str

Import always succeeds (so the CPU-only tests can import the package), but every compute call
raises ``ImportError`` when the compiled extension is missing: there is no CPU fallback.
Build in-tree with ``python fused-attention-cuda_b200/build.py``.
"""

from __future__ import annotations

import math

import torch
from torch import Tensor

from . import abi, ops, workloads

__all__ = [
    "__version__",
    "abi",
    "combine",
    "debug_set_skip_kv_tile",
    "forward",
    "forward_stage",
    "forward_strided",
    "impl_name",
    "impl_supports",
    "is_available",
    "last_device_error",
    "ops",
    "set_debug_overrides",
    "set_wait_timeout_ns",
    "workloads",
]
__version__ = "0.1.0"

_EXT_ERROR: ImportError | None
try:
    from . import _C  # noqa: F401  (loading the .so runs the TORCH_LIBRARY initialisers)
except ImportError as exc:  # pragma: no cover - depends on the build
    _EXT_ERROR = exc
else:
    _EXT_ERROR = None
    ops.register_fakes()

_BUILD_HINT = (
    "fused_attn._C is not built. From the repository root run\n"
    "  python fused-attention-cuda_b200/build.py\n"
    "(nvcc 12.8+ for sm_100a and a CUDA-enabled torch)."
)

_DTYPE_NAMES = {torch.float32: "fp32", torch.float16: "fp16", torch.bfloat16: "bf16"}


def is_available() -> bool:
    """True when the compiled extension imported."""
    return _EXT_ERROR is None


def _require_ext() -> None:
    if _EXT_ERROR is not None:
        raise ImportError(_BUILD_HINT) from _EXT_ERROR


def _resolve_scale(q: Tensor, scale: float | None) -> float:
    # PyTorch's SDPA default, decided in exactly one place (reference __init__.py:69-72).
    return float(1.0 / math.sqrt(q.shape[-1]) if scale is None else scale)


def forward(q: Tensor, k: Tensor, v: Tensor, is_causal: bool = False, scale: float | None = None,
            return_lse: bool = False):
    """Fused attention forward.  Returns ``o`` (the reference wrapper's return value), or
    ``(o, lse)`` with ``return_lse=True``; the raw op always returns both."""
    _require_ext()
    o, lse = torch.ops.fused_attn.forward(q, k, v, bool(is_causal), _resolve_scale(q, scale))
    return (o, lse) if return_lse else o


def forward_strided(q: Tensor, k: Tensor, v: Tensor, is_causal: bool = False,
                    scale: float | None = None, return_lse: bool = False):
    """``forward`` on [B, H, N, D] views with any strides whose head dim is contiguous (no
    counterpart in the reference, which needs contiguous inputs).  A GPT-style projection
    ``x[B, T, 3*H*D]`` splits into heads with ``view`` + ``transpose`` only, and the output has
    q's layout, so merging the heads back is a view as well::

        q, k, v = qkv.view(B, T, 3, H, D).permute(2, 0, 3, 1, 4)   # no copy
        o = fused_attn.forward_strided(q, k, v, is_causal=True)     # [B, H, T, D] view
        y = o.transpose(1, 2).reshape(B, T, H * D)                   # no copy
    """
    _require_ext()
    o, lse = torch.ops.fused_attn.forward_strided(q, k, v, bool(is_causal),
                                                  _resolve_scale(q, scale))
    return (o, lse) if return_lse else o


def combine(o_parts, lse_parts) -> tuple[Tensor, Tensor]:
    """Merge attention partials of the same queries over disjoint key sets (split-KV, ring /
    context-parallel attention): ``lse = ln sum exp(lse_i)``, ``o = sum exp(lse_i - lse) o_i``.
    ``o_parts``: contiguous [B, H, N, D] tensors, ``lse_parts``: fp32 [B, H, N] as returned by
    ``forward(..., return_lse=True)``.  Causal self-attention over a sequence split into chunks
    c = 0..S-1 is, chunk by chunk::

        parts = [fused_attn.forward(q[c], k[j], v[j], is_causal=(j == c), return_lse=True)
                 for j in range(c + 1)]
        o_c, lse_c = fused_attn.combine(*zip(*parts))
    """
    _require_ext()
    return torch.ops.fused_attn.combine(list(o_parts), list(lse_parts))


def forward_stage(q: Tensor, k: Tensor, v: Tensor, stage: int, is_causal: bool = False,
                  scale: float | None = None) -> tuple[Tensor, Tensor]:
    """Run one explicit stage (1..5); this build implements stage 5 on sm_100a."""
    _require_ext()
    return torch.ops.fused_attn.forward_stage(q, k, v, bool(is_causal), _resolve_scale(q, scale),
                                              int(stage))


def impl_supports(stage: int, dtype: torch.dtype, head_dim: int) -> bool:
    _require_ext()
    name = _DTYPE_NAMES.get(dtype)
    if name is None:
        return False
    return bool(torch.ops.fused_attn.impl_supports(int(stage), name, int(head_dim)))


def impl_name(stage: int) -> str:
    _require_ext()
    return str(torch.ops.fused_attn.impl_name(int(stage)))


def set_debug_overrides(block_m: int = 0, block_n: int = 0) -> None:
    """TEST-ONLY: force the tile sizes (0 = default).  block_m in {0, 128}, block_n in
    {0, 32, 64, 128}.  Process-global, not thread-safe: reset to (0, 0) afterwards."""
    _require_ext()
    torch.ops.fused_attn.set_debug_overrides(int(block_m), int(block_n))


def last_device_error() -> tuple[int, int]:
    """(cudaError_t, cause bits) of the kernel's bounded waits since the previous call;
    synchronises the current device.  cudaErrorLaunchTimeout (702) means a wait ran out."""
    _require_ext()
    return abi.last_device_error()


def set_wait_timeout_ns(ns: int) -> None:
    """Time limit of every device-side wait (default 2 s)."""
    _require_ext()
    abi.set_wait_timeout_ns(ns)


def debug_set_skip_kv_tile(tile: int) -> None:
    """TEST-ONLY fault injection: the producer skips the K load of key tile ``tile`` (-1 = off)."""
    _require_ext()
    abi.debug_set_skip_kv_tile(tile)
