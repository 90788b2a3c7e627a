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

With one GPU, step 3 writes the bf16 output directly and 4-5 are skipped.  Summing
fp32 partials and rounding once keeps the single bf16 rounding of :194.
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


class FullLayerSession:
    """Device buffers, weight shards and RoPE tables of one attention layer for one shape."""

    def __init__(self, S: int, *, B: int = 1, hidden: int = 4096, num_q_heads: int = 32, num_kv_heads: int = 8,
                 head_dim: int = 128, theta: float = kernels.ROPE_THETA, rank: int = 0, world: int = 1, group=None,
                 device=None):
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

    def set_weights(self, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, wo: torch.Tensor) -> None:
        """Full HF-layout weights (any device); this rank keeps its shard's slices."""
        for dst, src in zip((self.wq, self.wk, self.wv, self.wo), shard_weights(self.shard, wq, wk, wv, wo, self.d)):
            dst.copy_(src)

    def launches_per_step(self) -> int:
        return 3 if self.world == 1 else 4  # + the NCCL all-reduce kernel (not ours)

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
        reduce_partials(self.run_partial(), self.world, self.group)
        return kernels.cast_bf16(self.partial, out=self.out)

    def run_host(self, h_host: torch.Tensor, out_host: torch.Tensor) -> torch.Tensor:
        """h_host [B,S,hidden] / out_host [B,S,hidden]: bf16 CPU tensors (pinned for async copies)."""
        self.h.copy_(h_host, non_blocking=True)
        self.run_device()
        out_host.copy_(self.out, non_blocking=True)
        return out_host
