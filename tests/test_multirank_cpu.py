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

    from llama3_8b_attention_optimize_b200.layer import pipelined_row_reduce, reduce_cast_gather, reduce_partials, \
        row_chunks, shard_weights
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

        # 2b. the same reduction pipelined over row chunks (compute chunk, all-reduce it,
        # finish it), with the chunk boundaries on 128-row tiles: identical sums
        S2 = 300
        attn2 = torch.randn(32, S2, d, generator=g)
        local2 = attn2[sh.q_begin:sh.q_begin + sh.q_count].transpose(0, 1).reshape(S2, -1).double()
        chunks = row_chunks(S2, 4)
        # (row blocks multiplied separately: BLAS may block a different M differently)
        whole = torch.cat([local2[s0:s0 + n] @ swo.double().t() for s0, n in chunks])
        reduce_partials(whole, world)
        assert [c[0] for c in chunks] == [0, 128, 256] and sum(c[1] for c in chunks) == S2
        part = torch.full((S2, hidden), float("nan"), dtype=torch.float64)
        out = torch.full_like(part, float("nan"))
        order = []

        def compute(s0, n):
            order.append(("c", s0))
            part[s0:s0 + n] = local2[s0:s0 + n] @ swo.double().t()

        def finish(s0, n):
            order.append(("f", s0))
            out[s0:s0 + n] = part[s0:s0 + n]

        pipelined_row_reduce(part, chunks, compute, world, finish=finish)
        assert torch.equal(out, whole) and torch.equal(part, whole)
        assert order == [("c", 0), ("f", 0), ("c", 128), ("f", 128), ("c", 256), ("f", 256)]

        # 2c. reduce-scatter + round + all-gather == all-reduce then round (fp32 partials)
        pf = (local2[:256] @ swo.double().t()).float()
        ar = pf.clone()
        reduce_partials(ar, world)
        got = torch.empty(256, hidden, dtype=torch.bfloat16)
        reduce_cast_gather(pf, got, world)
        assert torch.equal(got, ar.to(torch.bfloat16))
        with pytest.raises(ValueError):
            reduce_cast_gather(pf[:255], got[:255], world)

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
