"""Drop-in for the reference's CPU_Baseline package, computed on the B200.

Mirrors CPU_Baseline/cpu_baseline of the reference repository:

* ``BenchmarkConfig`` / ``PRESETS`` / ``MODEL_REFERENCE``   -- config.py:8-91
* ``round_to_bf16``                                      -- bf16.py:6-14
* ``generate_qkv`` / ``prepare_operands``                -- attention.py:11-43 (same RNG recipe)
* ``gqa_attention``                                      -- attention.py:60-84: same arguments and
  result ([q_heads, seq_len, head_dim] float32 numpy), computed by the fused
  tcgen05 kernel in bf16 with fp32 accumulation (inputs are rounded to bf16)
* ``estimate_matmul_ops`` / ``estimate_softmax_ops`` / ``estimate_bytes_accessed`` -- metrics.py:22-40

The reference's ``gqa_attention_cpu`` has no RoPE; neither has ``gqa_attention``.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass

import numpy as np
import torch

from . import kernels

MODEL_REFERENCE = {
    "model_name": "Llama-3.1-8B",
    "num_attention_heads": 32,
    "num_key_value_heads": 8,
    "head_dim": 128,
    "gqa_group_size": 4,
    "datatype": "BF16",
}

PRESETS = {
    "small": dict(q_heads=4, kv_heads=1, seq_len=16, head_dim=128),
    "medium": dict(q_heads=8, kv_heads=2, seq_len=64, head_dim=128),
    "llama3_like_seq128": dict(q_heads=32, kv_heads=8, seq_len=128, head_dim=128),
    "llama3_like_seq256": dict(q_heads=32, kv_heads=8, seq_len=256, head_dim=128),
    "llama3_like_seq512": dict(q_heads=32, kv_heads=8, seq_len=512, head_dim=128),
}


@dataclass(frozen=True)
class BenchmarkConfig:
    q_heads: int = 32
    kv_heads: int = 8
    seq_len: int = 128
    head_dim: int = 128
    dtype: str = "fp32"
    causal: bool = True
    seed: int = 2026
    warmup: int = 5
    repeat: int = 30

    @property
    def group_size(self) -> int:
        return self.q_heads // self.kv_heads

    @property
    def dtype_bytes(self) -> int:
        return 2 if self.dtype == "bf16_emulated" else 4

    def validate(self) -> None:
        if self.q_heads <= 0 or self.kv_heads <= 0:
            raise ValueError("q_heads and kv_heads must be positive")
        if self.q_heads % self.kv_heads != 0:
            raise ValueError("q_heads must be divisible by kv_heads for GQA")
        if self.seq_len <= 0 or self.head_dim <= 0:
            raise ValueError("seq_len and head_dim must be positive")
        if self.dtype not in {"fp32", "bf16_emulated"}:
            raise ValueError("dtype must be fp32 or bf16_emulated")
        if self.warmup < 0:
            raise ValueError("warmup must be >= 0")
        if self.repeat <= 0:
            raise ValueError("repeat must be > 0")

    def to_dict(self) -> dict:
        d = asdict(self)
        d["group_size"] = self.group_size
        d["dtype_bytes"] = self.dtype_bytes
        d["model_reference"] = MODEL_REFERENCE
        return d

    @classmethod
    def from_preset(cls, preset: str, **kw) -> "BenchmarkConfig":
        if preset not in PRESETS:
            raise ValueError(f"unknown preset {preset!r}; valid presets: {', '.join(sorted(PRESETS))}")
        return cls(**PRESETS[preset], **kw)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bias = np.uint32(0x7FFF) + ((bits >> 16) & np.uint32(1))
    return ((bits + bias) & np.uint32(0xFFFF0000)).view(np.float32)


def prepare_operands(q: np.ndarray, k: np.ndarray, v: np.ndarray, config: BenchmarkConfig):
    q, k, v = (np.ascontiguousarray(t, dtype=np.float32) for t in (q, k, v))
    if q.shape != (config.q_heads, config.seq_len, config.head_dim):
        raise ValueError(f"q shape mismatch: expected {(config.q_heads, config.seq_len, config.head_dim)}, got {q.shape}")
    for name, t in (("k", k), ("v", v)):
        if t.shape != (config.kv_heads, config.seq_len, config.head_dim):
            raise ValueError(f"{name} shape mismatch: expected {(config.kv_heads, config.seq_len, config.head_dim)}, "
                             f"got {t.shape}")
    if config.dtype == "bf16_emulated":
        q, k, v = round_to_bf16(q), round_to_bf16(k), round_to_bf16(v)
    return q, k, v


def generate_qkv(config: BenchmarkConfig):
    rng = np.random.default_rng(config.seed)
    q = (rng.standard_normal((config.q_heads, config.seq_len, config.head_dim)) * 0.02).astype(np.float32)
    k = (rng.standard_normal((config.kv_heads, config.seq_len, config.head_dim)) * 0.02).astype(np.float32)
    v = (rng.standard_normal((config.kv_heads, config.seq_len, config.head_dim)) * 0.02).astype(np.float32)
    return prepare_operands(q, k, v, config)


def gqa_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, config: BenchmarkConfig, device=None) -> np.ndarray:
    """GQA core on the GPU: same contract as the reference's gqa_attention_cpu."""
    config.validate()
    dev = torch.device(device or "cuda")
    tq, tk, tv = (torch.from_numpy(np.ascontiguousarray(t, dtype=np.float32)).to(dev).to(torch.bfloat16).contiguous()
                  for t in (q, k, v))
    out = kernels.prefill(tq, tk, tv, causal=config.causal)
    res = out.float().cpu().numpy()
    if config.dtype == "bf16_emulated":
        res = round_to_bf16(res)
    return res


def estimate_matmul_ops(config: BenchmarkConfig) -> int:
    return int(4 * config.q_heads * config.seq_len * config.seq_len * config.head_dim)


def estimate_softmax_ops(config: BenchmarkConfig) -> int:
    return int(5 * config.q_heads * config.seq_len * config.seq_len)


def estimate_bytes_accessed(config: BenchmarkConfig) -> int:
    b = config.dtype_bytes
    q = config.q_heads * config.seq_len * config.head_dim
    kv = 2 * config.kv_heads * config.seq_len * config.head_dim
    s = config.q_heads * config.seq_len * config.seq_len
    return int((q + kv + 2 * s + q) * b)
