"""Pin the CPU oracle against the reference's own golden vectors (no GPU).

Fixtures (tests/golden/, made by tests/golden/make_fixtures.py):
* fpga_slice.npz -- the reference's committed hex goldens (KV group 0, 4 Q heads, 128 tokens)
* layer_s32.npz  -- stage dumps of the reference's run_full_attention on seeded inputs (32 heads)
"""
import math
import os

import numpy as np
import pytest

from oracle import cpu_port
from oracle import golden as g

HERE = os.path.dirname(os.path.abspath(__file__))


def _ulp(a, b):
    def key(w):
        w = w.astype(np.int64)
        return np.where(w & 0x8000, 0x8000 - (w & 0x7FFF), 0x8000 + w)
    return np.abs(key(a) - key(b))


@pytest.fixture(scope="module")
def fs():
    return dict(np.load(os.path.join(HERE, "golden", "fpga_slice.npz")))


@pytest.fixture(scope="module")
def layer():
    return dict(np.load(os.path.join(HERE, "golden", "layer_s32.npz")))


STAGES = ["q_after_rope", "k_after_rope", "scores_before_mask", "scores_after_mask",
          "softmax_weights", "attn_out_per_head"]


def test_fpga_slice_end_to_end_bit_exact(fs):
    st = g.stages(fs["q_before_rope"], fs["k_before_rope"], fs["v"])
    for key in STAGES:
        assert np.array_equal(st[key], fs[key]), key


def test_fpga_slice_each_stage_isolated(fs):
    assert np.array_equal(g.scores(fs["q_after_rope"], fs["k_after_rope"]), fs["scores_before_mask"])
    assert np.array_equal(g.mask_golden(fs["scores_before_mask"]), fs["scores_after_mask"])
    assert np.array_equal(g.softmax(fs["scores_after_mask"]), fs["softmax_weights"])
    assert np.array_equal(g.pv(fs["softmax_weights"], fs["v"]), fs["attn_out_per_head"])
    # the PV module's own vectors and the RoPE module's vectors are the same data
    assert np.array_equal(g.pv(fs["pv_softmax_weights"], fs["pv_v"]), fs["pv_attn_out"])
    assert np.array_equal(fs["rope_q_after"], fs["q_after_rope"])
    assert np.array_equal(fs["rope_k_after"], fs["k_after_rope"])
    assert np.array_equal(g.softmax(fs["softmax_input_scores"]), fs["softmax_expected_probs"])


def test_hls_mask_word_semantics(fs):
    out = g.attention_mask(fs["mask_raw_scores"], 4, 128, causal=True, mask_value=0xFF80)
    assert np.array_equal(out.reshape(4, 128, 128), fs["scores_after_mask"])
    # non-causal is a pure copy; the mask word is whatever the caller asks
    assert np.array_equal(g.attention_mask(fs["mask_raw_scores"], 4, 128, causal=False),
                          fs["mask_raw_scores"].reshape(-1))
    alt = g.attention_mask(fs["mask_raw_scores"], 4, 128, causal=True, mask_value=0xCE6E).reshape(4, 128, 128)
    iu = np.triu_indices(128, 1)
    assert np.all(alt[:, iu[0], iu[1]] == 0xCE6E)
    # the softmax module's mask file flags exactly the future (masked) positions
    flags = fs["softmax_input_masks"].reshape(4, 128, 128)
    for h in range(4):
        assert np.array_equal(flags[h], np.triu(np.ones((128, 128), np.uint16), 1))
    with pytest.raises(ValueError):
        g.attention_mask(fs["mask_raw_scores"], 0, 128)


def test_rope_tables_vs_reference_rom(fs):
    # The reference's sin/cos ROM words were built from float64 angles; the golden
    # model itself uses fp32 angles (its RoPE outputs match this oracle bit-exactly).
    cos, sin = g.rope_table(128)
    assert np.array_equal(cos[:, :64], cos[:, 64:])
    assert _ulp(cos[:, :64], fs["cos_pairs"]).max() <= 1
    assert _ulp(sin[:, :64], fs["sin_pairs"]).max() <= 2
    assert (_ulp(sin[:, :64], fs["sin_pairs"]) == 0).mean() > 0.999


def test_rope_table_matches_torch_recipe():
    """The oracle's (and the kernels') cos/sin tables against the golden's torch fp32
    recipe (llama3_attention_golden_model.py:124-130) over 32769 positions, the longest
    table the decode path builds.

    The oracle rounds cos/sin of each fp32 angle, evaluated in double precision, to fp32
    and then to bf16; torch evaluates them in fp32 with its own CPU math library.  The
    two agree on every word except where torch's fp32 result sits on (or one fp32 ulp
    from) the midpoint between two bf16 values, so that the fp32 evaluation decides the
    bf16 rounding.  Over 32769 x 128 words this happens at one angle (position 27067,
    pair 3: torch's fp32 sin is exactly -0.998046875, the midpoint, while the double
    value lies just inside it), i.e. two words, each one bf16 ulp apart.  The test
    requires exact agreement below position 8192 (every prefill configuration) and,
    beyond it, that every difference is one ulp at such a midpoint.
    """
    torch = pytest.importorskip("torch")
    S, D, theta = 32769, 128, 500000.0
    inv = 1.0 / (theta ** (torch.arange(0, D, 2).float() / D))
    assert np.array_equal(inv.numpy(), g.inv_freq(D, theta))
    emb = torch.outer(torch.arange(S).float(), inv)
    emb = torch.cat([emb, emb], dim=-1)
    cos, sin = g.rope_table(S, D, theta)
    n_diff = 0
    for fn, ours in ((torch.cos, cos), (torch.sin, sin)):
        f32 = fn(emb)
        ref = f32.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(ours[:8192], ref[:8192])
        bad = np.argwhere(ours != ref)
        n_diff += len(bad)
        for i, j in bad:
            assert _ulp(ours[i:i + 1, j], ref[i:i + 1, j]).max() == 1, (i, j)
            low = int(f32[i, j].view(torch.int32).item()) & 0xFFFF  # fp32 bits below the bf16 word
            assert abs(low - 0x8000) <= 1, (i, j, hex(low))
    assert n_diff <= 8, n_diff


def test_layer_fixture_all_stages_bit_exact(layer):
    st = g.stages(layer["q_before_rope"], layer["k_before_rope"], layer["v"])
    for key in STAGES:
        assert np.array_equal(st[key], layer[key]), key


def test_layer_fixture_gqa_mapping(layer):
    # q head h uses kv head h // 4: permuting KV heads must change exactly the mapped outputs
    q, k, v = layer["q_after_rope"], layer["k_after_rope"], layer["v"]
    base = g.pv(g.softmax(g.mask_golden(g.scores(q, k))), v)
    k2, v2 = k.copy(), v.copy()
    k2[3] = k[5]
    v2[3] = v[5]
    alt = g.pv(g.softmax(g.mask_golden(g.scores(q, k2))), v2)
    changed = [h for h in range(32) if not np.array_equal(base[h], alt[h])]
    assert changed == [12, 13, 14, 15]


def test_bf16_rounding_matches_cpu_baseline():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(100000) * 10).astype(np.float32)
    x[:4] = [0.0, -0.0, np.inf, -np.inf]
    words = g.to_bf16_words(x)
    assert np.array_equal(g.bf16_words_to_f32(words), cpu_port.round_to_bf16(x))


def test_attention_rows_matches_fp32_baseline(fs):
    # exact sampled-row attention == CPU_Baseline's fp32 core on the same (rotated) inputs
    q = g.bf16_words_to_f32(fs["q_after_rope"])
    k = g.bf16_words_to_f32(fs["k_after_rope"])
    v = g.bf16_words_to_f32(fs["v"])
    cfg = cpu_port.BaselineConfig(q_heads=4, kv_heads=1, seq_len=128, head_dim=128)
    ref = cpu_port.gqa_attention_cpu(q, k, v, cfg)
    heads = np.repeat(np.arange(4), 128)
    pos = np.tile(np.arange(128), 4)
    rows = g.attention_rows(fs["q_after_rope"], fs["k_after_rope"], fs["v"], heads, pos)
    assert np.abs(rows.reshape(4, 128, 128) - ref).max() < 2e-6
    # and the bf16-staged golden context is within the north-star tolerance of fp32
    ctx = g.bf16_words_to_f32(fs["attn_out_per_head"])
    assert np.abs(ctx - ref).max() < 1e-2 and np.abs(ctx - ref).mean() < 1e-3


def test_cpu_baseline_presets_and_validation():
    for name, p in cpu_port.PRESETS.items():
        cfg = cpu_port.BaselineConfig(**p)
        cfg.validate()
        assert cfg.group_size == p["q_heads"] // p["kv_heads"]
    with pytest.raises(ValueError):
        cpu_port.BaselineConfig(q_heads=6, kv_heads=4).validate()
    cfg = cpu_port.BaselineConfig(**cpu_port.PRESETS["small"])
    q, k, v = cpu_port.generate_qkv(cfg)
    out = cpu_port.gqa_attention_cpu(q, k, v, cfg)
    assert out.shape == (4, 16, 128) and np.isfinite(out).all()
    # row 0 attends only key 0
    np.testing.assert_allclose(out[:, 0], np.repeat(v[0:1, 0], 4, axis=0), rtol=0, atol=1e-7)
    assert cpu_port.estimate_matmul_ops(32, 128, 128) == 4 * 32 * 128 * 128 * 128
    assert cpu_port.causal_flops(4, 32, 8192, 128) == pytest.approx(2.1993e12, rel=1e-4)
    assert g.scale_for(128) == pytest.approx(1 / math.sqrt(128), rel=1e-7)
