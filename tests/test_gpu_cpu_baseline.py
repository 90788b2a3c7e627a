"""The CPU_Baseline drop-in (cpu_baseline.gqa_attention) against the reference's own
contract, gqa_attention_cpu (CPU_Baseline/cpu_baseline/attention.py:60-84), restated
by the oracle (oracle/cpu_port.py).

For every preset of config.py:19-25, with the reference's input recipe generate_qkv
(default_rng(seed), N(0,1) * 0.02, Q then K then V; attention.py:11-18), for dtype
fp32 and bf16_emulated and with the causal mask on and off:

* the facade's generate_qkv is bit-identical to the oracle's (a CPU test, below);
* every mode stays within the task's tolerance of the oracle: max-abs 1e-2, mean-abs
  1e-3;
* and, since the 0.02 input scale makes every output tiny, also within a bound scaled
  to the data: one bf16 ulp of the value (the output rounding) plus 2^-7 of the largest
  |v| (the softmax weights multiply V as bf16, so each weight is off by at most 2^-9 of
  itself: |sum_i dw_i (v_i - o)| <= 2^-8 * 2 max|v|).  fp32 compares with the oracle
  on the same bf16-rounded inputs (the facade rounds them, as the kernel computes in
  bf16) and, with twice that allowance, with the oracle on the unrounded inputs;
  bf16_emulated compares with the oracle's bf16_emulated result (rounded inputs, and
  the output rounded to bf16 as the reference does).
"""
import numpy as np
import pytest

from llama3_8b_attention_optimize_b200 import cpu_baseline as cb
from oracle import cpu_port

PRESETS = sorted(cb.PRESETS)


def _ulp(x: np.ndarray) -> np.ndarray:
    ax = np.maximum(np.abs(x).astype(np.float32), np.float32(2.0 ** -126))
    return np.exp2(np.floor(np.log2(ax)) - 7).astype(np.float32)


@pytest.mark.parametrize("preset", PRESETS)
@pytest.mark.parametrize("dtype", ["fp32", "bf16_emulated"])
def test_generate_qkv_matches_the_reference_recipe(preset, dtype):
    cfg = cb.BenchmarkConfig.from_preset(preset, dtype=dtype)
    ocfg = cpu_port.BaselineConfig(**cb.PRESETS[preset], dtype=dtype)
    for a, b in zip(cb.generate_qkv(cfg), cpu_port.generate_qkv(ocfg)):
        assert a.dtype == np.float32 and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("preset", PRESETS)
@pytest.mark.parametrize("dtype", ["fp32", "bf16_emulated"])
@pytest.mark.parametrize("causal", [True, False])
def test_gqa_attention_matches_gqa_attention_cpu(preset, dtype, causal):
    cfg = cb.BenchmarkConfig.from_preset(preset, dtype=dtype, causal=causal)
    ocfg = cpu_port.BaselineConfig(**cb.PRESETS[preset], dtype=dtype, causal=causal)
    q, k, v = cb.generate_qkv(cfg)
    got = cb.gqa_attention(q, k, v, cfg)
    assert got.shape == (cfg.q_heads, cfg.seq_len, cfg.head_dim) and got.dtype == np.float32
    ref = cpu_port.gqa_attention_cpu(q, k, v, ocfg)
    err = np.abs(got.astype(np.float64) - ref)
    assert err.max() <= 1e-2 and err.mean() <= 1e-3, (err.max(), err.mean())
    slack = 2.0 ** -7 * np.abs(v).max()
    if dtype == "fp32":
        assert np.all(err <= _ulp(ref) + 2 * slack), err.max()
        # exact attention of the same bf16 inputs: one rounding of the output away
        qb, kb, vb = (cpu_port.round_to_bf16(t) for t in (q, k, v))
        ref_b = cpu_port.gqa_attention_cpu(qb, kb, vb, ocfg)
        assert np.all(np.abs(got - ref_b) <= _ulp(ref_b) + slack)
    else:
        assert np.array_equal(got, cpu_port.round_to_bf16(got))  # output on bf16 values
        assert np.all(err <= _ulp(ref) + slack), err.max()


@pytest.mark.gpu
def test_gqa_attention_rejects_what_the_reference_rejects():
    with pytest.raises(ValueError):
        cb.gqa_attention(*cb.generate_qkv(cb.BenchmarkConfig(q_heads=4, kv_heads=1, seq_len=8)),
                         cb.BenchmarkConfig(q_heads=4, kv_heads=1, seq_len=8, dtype="fp16"))
