"""NumPy restatement of the reference's CPU baseline -- TEST INFRASTRUCTURE ONLY.

Follows CPU_Baseline/cpu_baseline of the reference repository:

* ``round_to_bf16``         -- bf16.py:6-14 (RNE bit trick on fp32 words)
* ``BaselineConfig``        -- config.py:28-60 (q_heads, kv_heads, seq_len, head_dim,
                               dtype in {fp32, bf16_emulated}, causal, seed)
* ``PRESETS``               -- config.py:19-25
* ``generate_qkv``          -- attention.py:11-18 (default_rng(seed), N(0,1)*0.02, Q then K then V)
* ``gqa_attention_cpu``     -- attention.py:46-84 (per-head loop, kv head = q head // group,
                               fp32 sgemm, triu mask to -inf, stable softmax, PV)
* ``estimate_matmul_ops``   -- metrics.py:22-24 (non-causal 4*Hq*S*S*d)

It is the fp32 reference for tolerance checks and the timed CPU baseline
(``bench.py --impl reference`` and the ``cpu_baseline`` leg), never a product path.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

PRESETS = {
    "small": dict(q_heads=4, kv_heads=1, seq_len=16, head_dim=128),
    "medium": dict(q_heads=8, kv_heads=2, seq_len=64, head_dim=128),
    "llama3_like_seq128": dict(q_heads=32, kv_heads=8, seq_len=128, head_dim=128),
    "llama3_like_seq256": dict(q_heads=32, kv_heads=8, seq_len=256, head_dim=128),
    "llama3_like_seq512": dict(q_heads=32, kv_heads=8, seq_len=512, head_dim=128),
}


@dataclass(frozen=True)
class BaselineConfig:
    q_heads: int = 32
    kv_heads: int = 8
    seq_len: int = 128
    head_dim: int = 128
    dtype: str = "fp32"
    causal: bool = True
    seed: int = 2026

    @property
    def group_size(self) -> int:
        return self.q_heads // self.kv_heads

    def validate(self) -> None:
        if self.q_heads <= 0 or self.kv_heads <= 0:
            raise ValueError("q_heads and kv_heads must be positive")
        if self.q_heads % self.kv_heads != 0:
            raise ValueError("q_heads must be divisible by kv_heads for GQA")
        if self.seq_len <= 0 or self.head_dim <= 0:
            raise ValueError("seq_len and head_dim must be positive")
        if self.dtype not in {"fp32", "bf16_emulated"}:
            raise ValueError("dtype must be fp32 or bf16_emulated")


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16 value, kept as fp32."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bias = np.uint32(0x7FFF) + ((bits >> 16) & np.uint32(1))
    return ((bits + bias) & np.uint32(0xFFFF0000)).view(np.float32)


def generate_qkv(cfg: BaselineConfig):
    rng = np.random.default_rng(cfg.seed)
    shp_q = (cfg.q_heads, cfg.seq_len, cfg.head_dim)
    shp_kv = (cfg.kv_heads, cfg.seq_len, cfg.head_dim)
    q = (rng.standard_normal(shp_q) * 0.02).astype(np.float32)
    k = (rng.standard_normal(shp_kv) * 0.02).astype(np.float32)
    v = (rng.standard_normal(shp_kv) * 0.02).astype(np.float32)
    if cfg.dtype == "bf16_emulated":
        q, k, v = round_to_bf16(q), round_to_bf16(k), round_to_bf16(v)
    return q, k, v


def _softmax_rows(s: np.ndarray) -> np.ndarray:
    m = np.max(s, axis=-1, keepdims=True)
    e = np.exp(s - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def gqa_attention_cpu(q: np.ndarray, k: np.ndarray, v: np.ndarray, cfg: BaselineConfig) -> np.ndarray:
    """fp32 GQA core: out[h] = softmax(mask(q[h] k[h//G]^T / sqrt(d))) v[h//G]."""
    cfg.validate()
    scale = 1.0 / math.sqrt(cfg.head_dim)
    out = np.empty((cfg.q_heads, cfg.seq_len, cfg.head_dim), dtype=np.float32)
    upper = np.triu(np.ones((cfg.seq_len, cfg.seq_len), dtype=bool), k=1) if cfg.causal else None
    for h in range(cfg.q_heads):
        g = h // cfg.group_size
        with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
            s = (q[h] @ k[g].T) * scale
        if upper is not None:
            s[upper] = -np.inf
        p = _softmax_rows(s).astype(np.float32, copy=False)
        with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
            o = p @ v[g]
        if cfg.dtype == "bf16_emulated":
            o = round_to_bf16(o)
        out[h] = o
    return out


def gqa_attention_head(q_h: np.ndarray, k_g: np.ndarray, v_g: np.ndarray, causal: bool = True) -> np.ndarray:
    """One head of ``gqa_attention_cpu`` (used for bounded CPU-baseline samples)."""
    S, d = q_h.shape
    s = (q_h @ k_g.T) * (1.0 / math.sqrt(d))
    if causal:
        s[np.triu(np.ones((S, k_g.shape[0]), dtype=bool), k=1)] = -np.inf
    return (_softmax_rows(s).astype(np.float32, copy=False) @ v_g).astype(np.float32)


def estimate_matmul_ops(q_heads: int, seq_len: int, head_dim: int) -> int:
    """Non-causal operation count of the reference's metrics (4*Hq*S*S*d)."""
    return int(4 * q_heads * seq_len * seq_len * head_dim)


def causal_flops(batch: int, q_heads: int, seq_len: int, head_dim: int) -> float:
    """Useful causal FLOPs: 4*B*Hq*d*S(S+1)/2 (QK^T and PV over the lower triangle)."""
    return 4.0 * batch * q_heads * head_dim * seq_len * (seq_len + 1) / 2.0
