"""The reference's main() flow on the B200 (llama3_attention_golden_model.py:201-249):
weights from safetensors, the seeded input, every stage, full/ and fpga_slice/ dumps,
then the fpga_slice hex files (prepare_attention_fpga_slice_vectors.py)."""
import os

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

from llama3_8b_attention_optimize_b200 import golden_model as gm
from llama3_8b_attention_optimize_b200 import hexio

pytestmark = pytest.mark.gpu


def test_main_writes_dumps_and_hex(tmp_path):
    g = torch.Generator().manual_seed(11)
    names = [f"model.layers.0.self_attn.{n}_proj.weight" for n in ("q", "k", "v", "o")]
    shapes = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096)]
    w = {n: (torch.randn(s, generator=g) * 0.02).to(torch.bfloat16) for n, s in zip(names, shapes)}
    wdir = tmp_path / "weights"
    wdir.mkdir()
    save_file(w, str(wdir / "model.safetensors"))
    out = tmp_path / "golden_model_outputs"
    dump = gm.main(str(wdir), str(out), seq_len=128)
    full = {f[:-4] for f in os.listdir(out / "full")}
    assert set(gm.STAGE_NAMES) <= full
    assert {"hidden_states_input", "q_proj", "k_proj", "v_proj", "o_proj"} <= full
    torch.manual_seed(42)
    h = gm.to_bf16(torch.randn(128, 4096) * 0.02)
    assert np.array_equal(np.load(out / "full" / "hidden_states_input.npy"), h.numpy())
    # the same computation through the facade directly is bit-identical
    again = gm.run_full_attention(h, *(w[n].float() for n in names))
    assert torch.equal(again["final_output"], dump["final_output"])
    assert torch.isfinite(dump["final_output"]).all() and dump["final_output"].shape == (128, 4096)
    man = hexio.prepare_from_npy(out / "fpga_slice", tmp_path / "tb")
    sl = gm.fpga_slice(dump)
    for npy_name, hex_name in hexio.NPY_TO_HEX.items():
        words = hexio.read_hex(tmp_path / "tb" / hex_name, int(np.prod(hexio.SHAPES[npy_name])))
        assert np.array_equal(words.reshape(hexio.SHAPES[npy_name]), hexio.bf16_words(sl[npy_name[:-4]]))
    assert len(man["outputs"]) == 9
