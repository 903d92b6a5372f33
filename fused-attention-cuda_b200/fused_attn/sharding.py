"""Head / batch sharding of the forward across the GPUs of one box (no hot-path collective).

Attention is independent per (batch, head), so a multi-GPU run partitions (b, h) pairs into
contiguous per-rank blocks and every rank runs the single-GPU kernel on its block; a head's
Q/K/V/O never leaves its GPU.  Collectives appear only off the hot path: the max-over-ranks
device time after timing, and an optional gather of O/LSE slices for checking.

The long-context configuration (C4: B1 H32 N16384 D128) splits its 32 heads into 32/k heads per
rank (strong scaling); the default benchmark gives every rank the same per-GPU workload on its
own batch shard (weak scaling).  With GQA the split is over kv-head groups, so each rank owns
whole groups and no K/V head is needed on two ranks.
"""

from __future__ import annotations

import torch


def head_range(num_heads: int, world: int, rank: int, hkv: int | None = None) -> tuple[int, int]:
    """[h0, h1) of the query heads owned by `rank`; whole kv groups when `hkv` < num_heads."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    hkv = num_heads if hkv is None else hkv
    if num_heads % hkv:
        raise ValueError(f"H={num_heads} must be a multiple of Hkv={hkv}")
    if hkv % world:
        raise ValueError(f"{hkv} kv heads cannot be split evenly over {world} ranks")
    group = num_heads // hkv
    per = hkv // world
    return rank * per * group, (rank + 1) * per * group


def kv_head_range(num_heads: int, world: int, rank: int, hkv: int | None = None) -> tuple[int, int]:
    hkv = num_heads if hkv is None else hkv
    h0, h1 = head_range(num_heads, world, rank, hkv)
    group = num_heads // hkv
    return h0 // group, h1 // group


def shard_heads(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, world: int, rank: int):
    """The rank's contiguous [B, H/world, N, D] (and kv) slices of full tensors."""
    h, hkv = q.shape[1], k.shape[1]
    h0, h1 = head_range(h, world, rank, hkv)
    k0, k1 = kv_head_range(h, world, rank, hkv)
    return (q[:, h0:h1].contiguous(), k[:, k0:k1].contiguous(), v[:, k0:k1].contiguous())


def batch_seed(base_seed: int, rank: int) -> int:
    """Seed of rank's batch shard in the weak-scaling run."""
    return base_seed + rank


def max_over_ranks(value: float, device: torch.device | str = "cpu", group=None) -> float:
    """All-reduce MAX of a per-rank time (off the hot path).  Single process: identity."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_heads(x: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather per-rank head slices [B, H/world, ...] back to [B, H, ...] (checking only)."""
    import torch.distributed as dist

    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return torch.cat(parts, dim=1)
