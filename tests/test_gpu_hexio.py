"""End-to-end GPU production of the reference's RTL test-bench vectors: from the slice's
input hex files, every stage runs on the B200 and the emitted hex files equal the
reference's committed ones byte for byte (SHA-256 from its manifest)."""
import json
import os

import numpy as np
import pytest

from llama3_8b_attention_optimize_b200 import hexio

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def fs():
    return dict(np.load(os.path.join(HERE, "golden", "fpga_slice.npz")))


@pytest.fixture(scope="module")
def sha():
    with open(os.path.join(HERE, "golden", "fpga_slice_sha256.json")) as f:
        return json.load(f)


def test_fpga_slice_from_hex_bit_exact(tmp_path, fs, sha):
    src = tmp_path / "in"
    src.mkdir()
    for npy_name, hex_name in hexio.NPY_TO_HEX.items():
        if npy_name in ("q_before_rope.npy", "k_before_rope.npy", "v.npy"):
            hexio.write_hex(src / hex_name, fs[npy_name[:-4]])
    out = tmp_path / "out"
    man = hexio.fpga_slice_from_hex(src, out)
    assert set(man["outputs"]) == set(hexio.NPY_TO_HEX.values()) | set(hexio.ROM_TABLES)
    for name in man["outputs"]:
        assert hexio.sha256(out / name) == sha[name], name


def test_fpga_slice_from_hex_checks_existing(tmp_path, fs):
    src = tmp_path / "in"
    src.mkdir()
    for npy_name, hex_name in hexio.NPY_TO_HEX.items():
        hexio.write_hex(src / hex_name, fs[npy_name[:-4]])
    hexio.fpga_slice_from_hex(src, tmp_path / "ok", existing=True)
    wrong = fs["attn_out_per_head"].copy()
    wrong.reshape(-1)[4097] ^= 0x10
    hexio.write_hex(src / "attn_out_per_head_bf16.hex", wrong)
    with pytest.raises(RuntimeError, match="at word 4097"):
        hexio.fpga_slice_from_hex(src, tmp_path / "bad", existing=True)
