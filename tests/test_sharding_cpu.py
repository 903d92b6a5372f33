"""Multi-process host logic of the head-sharded run, on CPU with the gloo backend.

* head_range / kv_head_range partition the heads contiguously (whole kv groups with GQA);
* world_size 2: each rank computes its head slice (with the CPU oracle standing in for the GPU
  kernel, which cannot run here) and the gathered result equals the unsharded computation;
* max_over_ranks returns the slowest rank's time;
* failure detection: a rank that raises before the collective (never joins) makes the other
  rank's collective end with an error within the process group's short timeout -- no hang.
"""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

from fused_attn.sharding import head_range, kv_head_range, shard_heads


def test_head_ranges_partition():
    for h, hkv, world in [(32, 32, 1), (32, 32, 2), (32, 32, 4), (32, 32, 8), (8, 2, 2), (12, 4, 4)]:
        seen = []
        for r in range(world):
            h0, h1 = head_range(h, world, r, hkv)
            seen.extend(range(h0, h1))
            k0, k1 = kv_head_range(h, world, r, hkv)
            assert all(hq // (h // hkv) in range(k0, k1) for hq in range(h0, h1))
        assert seen == list(range(h))
    with pytest.raises(ValueError):
        head_range(32, 3, 0)
    with pytest.raises(ValueError):
        head_range(8, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, out_q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import sys

        from conftest import PKG_DIR, ROOT  # noqa: F401  (sys.path set up by conftest import)

        for p in (str(PKG_DIR), str(ROOT)):
            if p not in sys.path:
                sys.path.insert(0, p)
        import torch.distributed as dist

        import oracle
        from fused_attn.sharding import gather_heads, max_over_ranks
        from fused_attn.workloads import make_qkv

        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5))
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the collective")
        q, k, v = make_qkv(1, 8, 64, 64, dtype=torch.float16, hkv=4, seed=3)
        qs, ks, vs = shard_heads(q, k, v, world, rank)
        o, lse = oracle.attention(qs, ks, vs, causal=True)
        o_all = gather_heads(torch.from_numpy(o), world)
        lse_all = gather_heads(torch.from_numpy(lse), world)
        slowest = max_over_ranks(1.0 + rank)
        if rank == 0:
            o_ref, lse_ref = oracle.attention(q, k, v, causal=True)
            out_q.put(("ok", float((o_all - torch.from_numpy(o_ref)).abs().max()),
                       float((lse_all - torch.from_numpy(lse_ref)).abs().max()), slowest))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent, never swallowed
        out_q.put(("error", rank, type(exc).__name__, str(exc)[:200], traceback.format_exc()[-400:]))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    results = []
    while not q.empty():
        results.append(q.get())
    return results, alive


def test_two_rank_head_sharding_matches_unsharded():
    results, alive = _run("ok")
    assert not alive
    oks = [r for r in results if r[0] == "ok"]
    assert oks, results
    _, eo, el, slowest = oks[0]
    assert eo == 0.0 and el == 0.0  # same fp64 arithmetic per head, gathered in order
    assert slowest == 2.0


def test_rank_failure_is_detected_not_hung():
    results, alive = _run("fail")
    assert not alive, "a rank hung instead of failing"
    errors = {r[1]: r for r in results if r[0] == "error"}
    assert 1 in errors and "fails before the collective" in errors[1][3]
    assert 0 in errors, f"rank 0 did not observe the failure: {results}"
