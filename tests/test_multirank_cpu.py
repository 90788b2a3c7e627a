"""Multi-rank host logic on CPU (gloo, world size 2): KV-head shard assignment, the
row-parallel o_proj reduction of the full layer, and the bench's max-over-ranks timing.

The GPU kernels are not called here (no device); the shard's partial product is
computed with torch on the CPU, which is all the reduction plumbing needs.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str):
    import sys
    sys.path.insert(0, ROOT)
    from datetime import timedelta

    from llama3_8b_attention_optimize_b200.layer import reduce_partials, shard_weights
    from llama3_8b_attention_optimize_b200.shard import kv_shard

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        # 1. every kv head is owned by exactly one rank, q heads follow their kv head
        sh = kv_shard(rank, world)
        shards = [None] * world
        dist.all_gather_object(shards, (sh.kv_begin, sh.kv_count, sh.q_begin, sh.q_count))
        kv = sorted(h for b, c, _, _ in shards for h in range(b, b + c))
        qh = sorted(h for _, _, b, c in shards for h in range(b, b + c))
        assert kv == list(range(8)) and qh == list(range(32))

        # 2. row-parallel o_proj: per-rank partials over the shard's q heads sum to the full product
        g = torch.Generator().manual_seed(3)  # same inputs on every rank
        S, hidden, d = 16, 4096, 128
        attn = torch.randn(32, S, d, generator=g)
        wq = torch.randn(4096, hidden, generator=g)
        wk = torch.randn(1024, hidden, generator=g)
        wv = torch.randn(1024, hidden, generator=g)
        wo = torch.randn(hidden, 4096, generator=g)
        swq, swk, swv, swo = shard_weights(sh, wq, wk, wv, wo)
        assert torch.equal(swq, wq[sh.q_begin * d:(sh.q_begin + sh.q_count) * d])
        assert torch.equal(swk, wk[sh.kv_begin * d:(sh.kv_begin + sh.kv_count) * d]) and swv.shape == swk.shape
        local = attn[sh.q_begin:sh.q_begin + sh.q_count].transpose(0, 1).reshape(S, -1).double()
        partial = local @ swo.double().t()
        reduce_partials(partial, world)
        full = attn.transpose(0, 1).reshape(S, -1).double() @ wo.double().t()
        assert torch.allclose(partial, full, rtol=1e-10, atol=1e-8)

        # 3. bench timing: the slowest rank's time is reported by every rank
        import bench
        t = bench.max_over_ranks(1.0 + rank, world, device="cpu")
        assert t == float(world)
        with open(os.path.join(out_dir, f"rank{rank}.ok"), "w") as f:
            f.write("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(240)
def test_two_rank_shards_reduction_and_timing(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    assert all((tmp_path / f"rank{r}.ok").exists() for r in range(world))
