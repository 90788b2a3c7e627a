"""KV-head sharding of the GQA core across the GPUs of one node.

The reference iterates over its 8 GQA groups sequentially in one chip
(FPT_BC_QK_Softmax_PV_Delivery_v5/doc/architecture.md:45-58; group -> kv head
mapping softmax_pv_backend/README.md:33-38).  Here each rank owns a contiguous
range of KV heads and the 4 query heads of each: the attention core needs no
communication, so ranks exchange nothing on the data path.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class KVShard:
    rank: int
    world: int
    kv_begin: int
    kv_count: int
    group: int  # query heads per kv head

    @property
    def q_begin(self) -> int:
        return self.kv_begin * self.group

    @property
    def q_count(self) -> int:
        return self.kv_count * self.group

    def q_heads(self) -> range:
        return range(self.q_begin, self.q_begin + self.q_count)

    def kv_heads(self) -> range:
        return range(self.kv_begin, self.kv_begin + self.kv_count)


def kv_shard(rank: int, world: int, num_kv_heads: int = 8, num_q_heads: int = 32) -> KVShard:
    """Contiguous, balanced split of the KV heads; every rank gets at least one head."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if num_q_heads % num_kv_heads:
        raise ValueError("q heads must be a multiple of kv heads")
    if world > num_kv_heads:
        raise ValueError(f"cannot shard {num_kv_heads} kv heads over {world} ranks")
    base, extra = divmod(num_kv_heads, world)
    begin = rank * base + min(rank, extra)
    count = base + (1 if rank < extra else 0)
    return KVShard(rank, world, begin, count, num_q_heads // num_kv_heads)


def all_shards(world: int, num_kv_heads: int = 8, num_q_heads: int = 32) -> list[KVShard]:
    return [kv_shard(r, world, num_kv_heads, num_q_heads) for r in range(world)]
