"""GPU parity of RoPE and the per-stage (debug dump) kernels: bit-exact against the
oracle and against the reference's golden vectors."""
import os

import numpy as np
import pytest
import torch

from llama3_8b_attention_optimize_b200 import golden_model, kernels
from oracle import golden as g
from tests._util import bf16_words, words_to_bf16

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def fs():
    return dict(np.load(os.path.join(HERE, "golden", "fpga_slice.npz")))


@pytest.fixture(scope="module")
def layer():
    return dict(np.load(os.path.join(HERE, "golden", "layer_s32.npz")))


@pytest.mark.parametrize("S,pos0", [(128, 0), (8192, 0), (300, 4000)])
def test_rope_cache_bit_exact(S, pos0):
    cos, sin = kernels.rope_cache(S, 128, 500000.0, pos0=pos0)
    oc, osn = g.rope_table(S, 128, 500000.0, pos0=pos0)
    assert np.array_equal(bf16_words(cos), oc)
    assert np.array_equal(bf16_words(sin), osn)


def test_rope_apply_bit_exact_on_golden(fs):
    cos, sin = kernels.rope_cache(128)
    q = kernels.rope(words_to_bf16(fs["q_before_rope"]), cos, sin)
    k = kernels.rope(words_to_bf16(fs["k_before_rope"]), cos, sin)
    assert np.array_equal(bf16_words(q), fs["q_after_rope"])
    assert np.array_equal(bf16_words(k), fs["k_after_rope"])


def test_rope_in_place_and_offset():
    x = torch.randn(3, 40, 128, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).cuda()
    cos, sin = kernels.rope_cache(100)
    y = kernels.rope(x, cos, sin, pos0=60)
    oc, osn = g.rope_table(100)
    ref = g.rope_apply(bf16_words(x), oc[60:100], osn[60:100])
    assert np.array_equal(bf16_words(y), ref)
    x2 = x.clone()
    kernels.rope(x2, cos, sin, pos0=60, out=x2)
    assert torch.equal(x2, y)


def test_debug_stages_bit_exact_fpga_slice(fs):
    dump = golden_model.run_attention_core(torch.from_numpy(g.bf16_words_to_f32(fs["q_before_rope"])),
                                           torch.from_numpy(g.bf16_words_to_f32(fs["k_before_rope"])),
                                           torch.from_numpy(g.bf16_words_to_f32(fs["v"])), debug=True)
    for key in ("q_after_rope", "k_after_rope", "scores_before_mask", "scores_after_mask", "softmax_weights",
                "attn_out_per_head"):
        got = g.to_bf16_words(dump[key].numpy())
        assert np.array_equal(got, fs[key]), key


def test_debug_stages_bit_exact_layer(layer):
    q, k, v = (torch.from_numpy(g.bf16_words_to_f32(layer[n])) for n in ("q_before_rope", "k_before_rope", "v"))
    dump = golden_model.run_attention_core(q, k, v, debug=True)
    for key in ("q_after_rope", "k_after_rope", "scores_before_mask", "scores_after_mask", "softmax_weights",
                "attn_out_per_head"):
        assert np.array_equal(g.to_bf16_words(dump[key].numpy()), layer[key]), key


def test_hls_mask_words_bit_exact(fs):
    raw = torch.from_numpy(fs["mask_raw_scores"].reshape(-1).view(np.int16)).cuda()
    out = kernels.attention_mask_words(raw, 4, 128, causal=True)
    assert np.array_equal(out.cpu().numpy().view(np.uint16).reshape(4, 128, 128), fs["scores_after_mask"])
    out2 = kernels.attention_mask_words(raw, 4, 128, causal=False)
    assert torch.equal(out2, raw)
    out3 = kernels.attention_mask_words(raw, 4, 128, causal=True, mask_value=0xCE6E)
    ref3 = g.attention_mask(fs["mask_raw_scores"], 4, 128, True, 0xCE6E)
    assert np.array_equal(out3.cpu().numpy().view(np.uint16), ref3)


@pytest.mark.parametrize("S", [1, 17, 64, 130])
def test_stage_kernels_odd_sizes(S):
    rng = np.random.default_rng(S)
    q = g.to_bf16_words(rng.standard_normal((8, S, 128)).astype(np.float32))
    k = g.to_bf16_words(rng.standard_normal((2, S, 128)).astype(np.float32))
    v = g.to_bf16_words(rng.standard_normal((2, S, 128)).astype(np.float32))
    st = g.stages(q, k, v)
    dump = golden_model.run_attention_core(*(torch.from_numpy(g.bf16_words_to_f32(t)) for t in (q, k, v)))
    for key in ("q_after_rope", "scores_before_mask", "scores_after_mask", "softmax_weights", "attn_out_per_head"):
        assert np.array_equal(g.to_bf16_words(dump[key].numpy()), st[key]), (key, S)


def test_golden_facade_build_rope_cache_matches_reference_recipe():
    cos, sin = golden_model.build_rope_cache(256, 128, 500000.0)
    oc, osn = g.rope_table(256)
    assert cos.device.type == "cpu" and cos.dtype == torch.float32
    assert np.array_equal(g.to_bf16_words(cos.numpy()), oc)
    assert np.array_equal(g.to_bf16_words(sin.numpy()), osn)
