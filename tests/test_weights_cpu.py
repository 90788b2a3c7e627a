"""Layer-0 weight loading from safetensors (the reference's get_layer0_weight_paths /
load_layer0_weights, llama3_attention_golden_model.py:59-121): sharded index, single
file, missing entries, bf16 rounding.  No GPU, no network."""
import json

import pytest
import torch
from safetensors.torch import save_file

from llama3_8b_attention_optimize_b200 import golden_model as gm

NAMES = [f"model.layers.0.self_attn.{n}_proj.weight" for n in ("q", "k", "v", "o")]


def _weights(seed=3, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    shapes = [(64, 32), (16, 32), (16, 32), (32, 64)]
    return {n: (torch.randn(s, generator=g) * 0.02).to(dtype) for n, s in zip(NAMES, shapes)}


def test_sharded_index(tmp_path):
    w = _weights()
    save_file({NAMES[0]: w[NAMES[0]], NAMES[1]: w[NAMES[1]], "model.embed_tokens.weight": torch.zeros(4, 4)},
              str(tmp_path / "model-00001-of-00002.safetensors"))
    save_file({NAMES[2]: w[NAMES[2]], NAMES[3]: w[NAMES[3]]}, str(tmp_path / "model-00002-of-00002.safetensors"))
    wm = {NAMES[0]: "model-00001-of-00002.safetensors", NAMES[1]: "model-00001-of-00002.safetensors",
          NAMES[2]: "model-00002-of-00002.safetensors", NAMES[3]: "model-00002-of-00002.safetensors"}
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wm}))
    paths = gm.get_layer0_weight_paths(str(tmp_path))
    assert paths == {n: str(tmp_path / wm[n]) for n in NAMES}
    got = gm.load_layer0_weights(str(tmp_path))
    for t, n in zip(got, NAMES):
        assert t.dtype == torch.float32 and torch.equal(t, w[n].float())


def test_single_file_and_rounding(tmp_path):
    w = _weights(dtype=torch.float32)  # fp32 checkpoint: rounded to bf16 like the reference's to_bf16
    save_file(w, str(tmp_path / "model.safetensors"))
    assert set(gm.get_layer0_weight_paths(str(tmp_path)).values()) == {str(tmp_path / "model.safetensors")}
    got = gm.load_layer0_weights(str(tmp_path))
    for t, n in zip(got, NAMES):
        assert torch.equal(t, w[n].to(torch.bfloat16).float())


def test_missing_entries(tmp_path):
    w = _weights()
    save_file({n: w[n] for n in NAMES[:3]}, str(tmp_path / "model.safetensors"))
    with pytest.raises(KeyError, match="o_proj"):
        gm.load_layer0_weights(str(tmp_path))
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {NAMES[0]: "x"}}))
    with pytest.raises(KeyError, match="no entry"):
        gm.get_layer0_weight_paths(str(tmp_path))
