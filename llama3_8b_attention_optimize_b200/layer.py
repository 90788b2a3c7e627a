"""One Llama-3 attention layer on a KV-head shard (reference run_full_attention,
llama3_attention_golden_model.py:144-197, as one fused pipeline).

Per step, on every rank (rank r owns kv heads [g0, g0+c) and q heads [4g0, 4(g0+c))):

  1. gqa_qkv_proj_bf16   q, k, v = bf16(h @ W^T) head-major, q/k rotated in the
                         epilogue (column-parallel: only the shard's weight rows)
  2. gqa_prefill_bf16    causal GQA core on the shard's heads (no communication)
  3. gqa_o_proj_bf16     o_proj partial over the shard's q heads (row-parallel:
                         the shard's weight columns), fp32 when world > 1
  4. all-reduce (sum)    NCCL over NVLink / NVSwitch (world > 1 only)
  5. gqa_cast_f32_bf16   one rounding of the summed partials (world > 1 only)

``reduce="p2p"`` replaces 4-5 by an exchange through NVLink peer memory (no NCCL in the
step): the o_proj partial goes straight into a CUDA-IPC buffer every rank maps
(``PeerExchange``), each rank sums its row block of all partials by P2P loads, rounds
once and gathers the other blocks (``gqa_tp_reduce_gather_bf16``).

``reduce="p2p_fused"`` goes one step further: the o_proj GEMM's epilogue stores each fp32
row straight into the owning rank's buffer (NVLink stores while other tiles compute), and
the owners reduce, round and store their bf16 blocks into every rank's output
(``gqa_tp_o_proj_exchange_bf16``).

``reduce="rs_ag"`` replaces 4-5 by a reduce-scatter of the fp32 partials (each rank sums
S/world rows), the rounding of those rows, and an all-gather of the bf16 rows: the same
one rounding of the fp32 sum, with 3/4 of the all-reduce's bytes on the links.

With one GPU, step 3 writes the bf16 output directly and 4-5 are skipped.  Summing
fp32 partials and rounding once keeps the single bf16 rounding of :194.

With ``o_chunks`` > 1 (one sequence), steps 3-5 run as a pipeline over row chunks: the
GEMM of chunk i+1 (on the compute stream, grid capped to leave SMs for NCCL) overlaps the
all-reduce and the rounding of chunk i (on a communication stream).  Every row is
computed exactly as in the unchunked step.
"""
from __future__ import annotations

import torch

from . import kernels
from .shard import KVShard, kv_shard


def layer_flops(B: int, S: int, hidden: int = 4096, num_q_heads: int = 32, num_kv_heads: int = 8,
                head_dim: int = 128, causal: bool = True) -> dict:
    """Algorithmic FLOPs of one layer: projections (2 per MAC) and the attention core."""
    qkv = 2.0 * B * S * hidden * (num_q_heads + 2 * num_kv_heads) * head_dim
    o = 2.0 * B * S * (num_q_heads * head_dim) * hidden
    core = (4.0 * B * num_q_heads * head_dim * S * (S + 1) / 2.0 if causal
            else 4.0 * B * num_q_heads * head_dim * S * S)
    return {"qkv": qkv, "o_proj": o, "core": core, "total": qkv + o + core}


def shard_weights(shard: KVShard, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, wo: torch.Tensor,
                  head_dim: int = 128):
    """The rows of q/k/v_proj and the columns of o_proj that one shard multiplies with."""
    q0, q1 = shard.q_begin * head_dim, (shard.q_begin + shard.q_count) * head_dim
    k0, k1 = shard.kv_begin * head_dim, (shard.kv_begin + shard.kv_count) * head_dim
    return wq[q0:q1], wk[k0:k1], wv[k0:k1], wo[:, q0:q1]


def reduce_partials(partial: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """Sum the row-parallel o_proj partials of all ranks in place (identity for one rank).

    Every rank calls this once per step, in the same order (a collective)."""
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial


def row_chunks(S: int, n_chunks: int, align: int = 128) -> list:
    """Split rows [0, S) into up to n_chunks contiguous (s0, count) ranges whose starts are
    multiples of ``align`` (GEMM tile rows), as even as that allows."""
    if S <= 0 or n_chunks <= 0:
        raise ValueError("row_chunks needs S > 0 and n_chunks > 0")
    tiles = (S + align - 1) // align
    n = min(n_chunks, tiles)
    bounds = [min(S, ((i * tiles) // n) * align) for i in range(n)] + [S]
    return [(bounds[i], bounds[i + 1] - bounds[i]) for i in range(n) if bounds[i + 1] > bounds[i]]


def reduce_cast_gather(partial: torch.Tensor, out: torch.Tensor, world: int, group=None,
                       mine: torch.Tensor | None = None, cast=None) -> torch.Tensor:
    """out = bf16(sum over ranks of partial) via reduce-scatter (fp32 rows [S/world] per
    rank), the rounding of this rank's rows and an all-gather of the bf16 rows.
    partial [..., N] fp32 and out [..., N] bf16, the leading dimensions flattened to rows
    (a multiple of the world size); ``cast`` rounds
    fp32 -> bf16 (default: torch's round-to-nearest-even)."""
    import torch.distributed as dist

    n = partial.shape[-1]
    rows = partial.numel() // n  # all leading dimensions are rows
    if rows % world:
        raise ValueError("reduce_cast_gather needs rows divisible by the world size")
    p2 = partial.reshape(rows, n)
    o2 = out.reshape(rows, n)
    if mine is None:
        mine = torch.empty(rows // world, p2.shape[1], dtype=partial.dtype, device=partial.device)
    dist.reduce_scatter_tensor(mine, p2, op=dist.ReduceOp.SUM, group=group)
    mine_bf = cast(mine) if cast is not None else mine.to(out.dtype)
    dist.all_gather_into_tensor(o2, mine_bf, group=group)
    return out


class _DevArray:
    """A raw device allocation seen as a torch tensor (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """One CUDA-IPC buffer per rank ([partial fp32 S x N][out bf16 S x N][flags]) mapped by
    every other rank, for the NVLink-peer reduction of row-parallel partials.

    Construction is collective (handles travel by ``all_gather_object`` on ``group``);
    ``close()`` is collective too (a barrier, so no rank frees memory a peer still reads).
    """

    def __init__(self, S: int, N: int, rank: int, world: int, group=None, device=None):
        import ctypes

        import torch.distributed as dist

        from . import _lib

        lib = _lib.load()
        self.lib, self.S, self.N, self.rank, self.world, self.group = lib, S, N, rank, world, group
        self.device = torch.device(device or "cuda")
        nbytes = lib.gqa_tp_buffer_bytes(S, N)
        hb = lib.gqa_peer_handle_bytes()
        handle = ctypes.create_string_buffer(hb)
        ptr = ctypes.c_void_p()
        kernels.check(lib.gqa_peer_alloc(nbytes, ctypes.byref(ptr), handle), "gqa_peer_alloc")
        self._own = ptr.value
        handles = [None] * world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._opened = []
        bases = []
        err = ""
        for r, h in enumerate(handles):
            if r == rank:
                bases.append(self._own)
                continue
            pp = ctypes.c_void_p()
            rc = lib.gqa_peer_open(ctypes.create_string_buffer(h, hb), ctypes.byref(pp))
            if rc != 0:
                err = f"rank {rank}: gqa_peer_open of rank {r}'s buffer failed ({rc})"
                break
            self._opened.append(pp.value)
            bases.append(pp.value)
        # every rank learns whether every rank could map every peer, so all raise together
        errs = [None] * world
        dist.all_gather_object(errs, err, group=group)
        if any(errs):
            for pp in self._opened:
                lib.gqa_peer_close(pp)
            dist.barrier(group=group)
            lib.gqa_peer_free(self._own)
            raise RuntimeError("peer exchange unavailable: " + "; ".join(e for e in errs if e))
        self._bases = (ctypes.c_void_p * world)(*bases)
        self.partial = torch.as_tensor(_DevArray(self._own, (S, N), "<f4"), device=self.device)
        self.out = torch.as_tensor(_DevArray(self._own + S * N * 4, (S, N), "<i2"),
                                   device=self.device).view(torch.bfloat16)
        self.epoch = 0
        dist.barrier(group=group)

    def reduce_gather(self) -> torch.Tensor:
        """Sum the ranks' partials (the caller has written this rank's into ``partial``),
        round once, and return the full bf16 result in ``out``."""
        self.epoch += 1
        kernels.check(self.lib.gqa_tp_reduce_gather_bf16(self._bases, self.world, self.rank, self.S, self.N,
                                                         self.epoch, kernels._stream(self.device)),
                      "gqa_tp_reduce_gather_bf16")
        return self.out

    def o_proj_exchange(self, attn: torch.Tensor, wo: torch.Tensor) -> torch.Tensor:
        """The o_proj of attn [Hq, S, 128] (this rank's heads) against wo [N, Hq*128]
        fused with the exchange: rows go straight to their owners over NVLink; returns
        the full bf16 result in ``out``."""
        self.epoch += 1
        Hq = attn.shape[-3]
        kernels.check(self.lib.gqa_tp_o_proj_exchange_bf16(kernels._ptr(attn), kernels._ptr(wo), wo.shape[1],
                                                           self._bases, self.world, self.rank, self.S, Hq, 128,
                                                           self.N, self.epoch, kernels._stream(self.device)),
                      "gqa_tp_o_proj_exchange_bf16")
        return self.out

    def close(self) -> None:
        import torch.distributed as dist

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every rank is done reading every buffer
        for pp in self._opened:
            self.lib.gqa_peer_close(pp)
        self._opened = []
        dist.barrier(group=self.group)
        self.lib.gqa_peer_free(self._own)
        self._own = None


def pipelined_row_reduce(partial: torch.Tensor, chunks: list, compute, world: int, group=None, finish=None,
                         comm_stream=None) -> torch.Tensor:
    """For each row chunk: compute(s0, n) fills partial[s0:s0+n] on the current stream;
    the chunk is then summed across ranks (all-reduce) and passed to finish(s0, n) on
    ``comm_stream`` (when given, a CUDA stream that runs beside the next compute).  All
    ranks issue the same collectives in the same order.  Returns ``partial``."""
    import torch.distributed as dist

    cur = torch.cuda.current_stream(partial.device) if partial.is_cuda else None
    for s0, n in chunks:
        compute(s0, n)
        rows = partial.narrow(0, s0, n)
        if comm_stream is not None:
            comm_stream.wait_stream(cur)
            with torch.cuda.stream(comm_stream):
                if world > 1:
                    dist.all_reduce(rows, op=dist.ReduceOp.SUM, group=group)
                if finish is not None:
                    finish(s0, n)
        else:
            if world > 1:
                dist.all_reduce(rows, op=dist.ReduceOp.SUM, group=group)
            if finish is not None:
                finish(s0, n)
    if comm_stream is not None:
        cur.wait_stream(comm_stream)
    return partial


class FullLayerSession:
    """Device buffers, weight shards and RoPE tables of one attention layer for one shape."""

    def __init__(self, S: int, *, B: int = 1, hidden: int = 4096, num_q_heads: int = 32, num_kv_heads: int = 8,
                 head_dim: int = 128, theta: float = kernels.ROPE_THETA, rank: int = 0, world: int = 1, group=None,
                 device=None, o_chunks: int = 1, gemm_ctas: int = 0, reduce: str = "all_reduce"):
        self.device = torch.device(device or "cuda")
        self.shard = kv_shard(rank, world, num_kv_heads, num_q_heads)
        self.world, self.group = world, group
        self.B, self.S, self.hidden, self.d = B, S, hidden, head_dim
        self.num_q_heads, self.num_kv_heads = num_q_heads, num_kv_heads
        hq, hkv = self.shard.q_count, self.shard.kv_count
        mk = lambda *shp, dt=torch.bfloat16: torch.empty(shp, dtype=dt, device=self.device)  # noqa: E731
        self.h = mk(B, S, hidden)
        self.wq, self.wk, self.wv = mk(hq * head_dim, hidden), mk(hkv * head_dim, hidden), mk(hkv * head_dim, hidden)
        self.wo = mk(hidden, hq * head_dim)
        self.q, self.k, self.v = mk(B, hq, S, head_dim), mk(B, hkv, S, head_dim), mk(B, hkv, S, head_dim)
        self.attn = mk(B, hq, S, head_dim)
        self.partial = mk(B, S, hidden, dt=torch.float32) if world > 1 else None
        self.out = mk(B, S, hidden)
        self.cos, self.sin = kernels.rope_cache(S, head_dim, theta, device=self.device)
        # o_proj / all-reduce pipeline (one sequence, several ranks)
        self.o_chunks = o_chunks if (world > 1 and B == 1) else 1
        self.gemm_ctas = gemm_ctas
        self.chunks = row_chunks(S, self.o_chunks)
        self.comm_stream = torch.cuda.Stream(self.device) if self.o_chunks > 1 else None
        if reduce not in ("all_reduce", "rs_ag", "p2p", "p2p_fused"):
            raise ValueError("reduce must be 'all_reduce', 'rs_ag', 'p2p' or 'p2p_fused'")
        self.reduce = reduce if (world > 1 and (B * S) % world == 0) else "all_reduce"
        self.peer = None
        if self.reduce in ("p2p", "p2p_fused"):
            if B != 1:
                raise ValueError("reduce='p2p' takes one sequence")
            if self.reduce == "p2p_fused" and ((S // world) % 128 or hidden % 256):
                raise ValueError("reduce='p2p_fused' needs S / world to be a multiple of 128 rows and hidden a "
                                 "multiple of 256 (the o_proj tiles each rank stores into its owners)")
            self.peer = PeerExchange(S, hidden, rank, world, group, self.device)
            self.partial, self.out = self.peer.partial.view(B, S, hidden), self.peer.out.view(B, S, hidden)
        self._mine = (mk(B * S // world, hidden, dt=torch.float32) if self.reduce == "rs_ag" else None)
        self._mine_bf = (mk(B * S // world, hidden) if self.reduce == "rs_ag" else None)

    def set_weights(self, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, wo: torch.Tensor) -> None:
        """Full HF-layout weights (any device); this rank keeps its shard's slices."""
        for dst, src in zip((self.wq, self.wk, self.wv, self.wo), shard_weights(self.shard, wq, wk, wv, wo, self.d)):
            dst.copy_(src)

    def launches_per_step(self) -> int:
        if self.world == 1:
            return 3
        return 2 + 2 * len(self.chunks)  # o_proj and cast per chunk (+ NCCL all-reduces, not ours)

    def flops(self) -> dict:
        return layer_flops(self.B, self.S, self.hidden, self.num_q_heads, self.num_kv_heads, self.d)

    def _core(self) -> None:
        kernels.qkv_proj(self.h, self.wq, self.wk, self.wv, self.cos, self.sin, rope_q=True, rope_k=True,
                         head_dim=self.d, out=(self.q, self.k, self.v))
        kernels.prefill(self.q, self.k, self.v, causal=True, out=self.attn)

    def run_partial(self) -> torch.Tensor:
        """Steps 1-3 on a sharded session: this rank's fp32 o_proj partial (not yet reduced)."""
        if self.partial is None:
            raise RuntimeError("a single-rank session has no partials")
        self._core()
        return kernels.o_proj(self.attn, self.wo, out_f32=True, out=self.partial)

    def run_device(self) -> torch.Tensor:
        if self.world == 1:
            self._core()
            return kernels.o_proj(self.attn, self.wo, out=self.out)
        if self.reduce == "p2p":
            self.run_partial()
            self.peer.reduce_gather()
            return self.out
        if self.reduce == "p2p_fused":
            self._core()
            self.peer.o_proj_exchange(self.attn[0], self.wo)
            return self.out
        if self.reduce == "rs_ag":
            self.run_partial()
            return reduce_cast_gather(self.partial, self.out, self.world, self.group, mine=self._mine,
                                      cast=lambda x: kernels.cast_bf16(x, out=self._mine_bf))
        if self.o_chunks == 1:
            reduce_partials(self.run_partial(), self.world, self.group)
            return kernels.cast_bf16(self.partial, out=self.out)
        self._core()
        part, out = self.partial[0], self.out[0]

        def compute(s0, n):
            kernels.o_proj_rows(self.attn[0], self.wo, part, s0, n, out_f32=True, max_ctas=self.gemm_ctas)

        def finish(s0, n):
            kernels.cast_bf16(part.narrow(0, s0, n), out=out.narrow(0, s0, n))

        pipelined_row_reduce(part, self.chunks, compute, self.world, self.group, finish, self.comm_stream)
        return self.out

    def close(self) -> None:
        """Release the peer-memory exchange (collective when reduce='p2p')."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def run_host(self, h_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        """h_host [B,S,hidden] / out_host [B,S,hidden]: bf16 CPU tensors (pinned for async copies)."""
        self.h.copy_(h_host, non_blocking=True)
        self.run_device()
        out_host.copy_(self.out, non_blocking=True)
        return out_host
