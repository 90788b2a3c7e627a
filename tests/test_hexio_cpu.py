"""Hex fixture I/O (the reference's RTL test-bench vector format) on the CPU: the
writer and the RoPE ROM tables reproduce the reference's committed files byte for
byte (SHA-256 from its manifest), and the readers reject what the reference rejects."""
import hashlib
import json
import os

import numpy as np
import pytest

from llama3_8b_attention_optimize_b200 import hexio

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def fs():
    return dict(np.load(os.path.join(HERE, "golden", "fpga_slice.npz")))


@pytest.fixture(scope="module")
def sha():
    with open(os.path.join(HERE, "golden", "fpga_slice_sha256.json")) as f:
        return json.load(f)


def _f32(words):
    return (words.astype(np.uint32) << np.uint32(16)).view(np.float32)


def test_emit_matches_reference_files(tmp_path, fs, sha):
    arrays = {name: _f32(fs[name[:-4]]) for name in hexio.SHAPES}
    man = hexio.emit_fpga_slice(arrays, tmp_path)
    assert set(man["outputs"]) == set(hexio.NPY_TO_HEX.values()) | set(hexio.ROM_TABLES)
    for name, entry in man["outputs"].items():
        assert entry["sha256"] == sha[name], name
        assert hexio.sha256(tmp_path / name) == sha[name]
    saved = json.loads((tmp_path / hexio.MANIFEST_NAME).read_text())
    assert saved["configuration"]["seq_len"] == 128 and saved["outputs"] == man["outputs"]


def test_rope_rom_words_full_table(fs, sha):
    s, c = hexio.rope_rom_words(8192)
    assert s.shape == (8192, 64)
    assert np.array_equal(s[:128], fs["sin_pairs"]) and np.array_equal(c[:128], fs["cos_pairs"])
    for name, w in (("sin", s), ("cos", c)):
        assert hashlib.sha256(w.astype("<u2").tobytes()).hexdigest() == sha[f"rom_{name}_words"]
    s2, c2 = hexio.rope_rom_words(100, pos0=8000)
    assert np.array_equal(s2, s[8000:8100]) and np.array_equal(c2, c[8000:8100])


def test_read_write_round_trip_and_format(tmp_path, fs):
    p = tmp_path / "v.hex"
    hexio.write_hex(p, fs["v"])
    raw = p.read_bytes()
    assert raw.count(b"\n") == 16384 and b"\r" not in raw and raw[:5] == b"%04X\n" % int(fs["v"].reshape(-1)[0])
    assert np.array_equal(hexio.read_hex(p, 16384).reshape(1, 128, 128), fs["v"])
    # CRLF, lower case and blank lines are accepted on read
    q = tmp_path / "crlf.hex"
    q.write_bytes(b"00ff\r\n\r\n7FC0\r\n")
    assert list(hexio.read_hex(q, 2)) == [0x00FF, 0x7FC0]


@pytest.mark.parametrize("text,msg", [(b"12G4\n", "line 1: '12G4' is not a 16-bit hex word"),
                                      (b"0001\n\n1FFFF\n", "line 3: '1FFFF' is not a 16-bit hex word"),
                                      (b"0001\n0002\n", "2 words, want 3")])
def test_read_hex_rejects(tmp_path, text, msg):
    p = tmp_path / "bad.hex"
    p.write_bytes(text)
    with pytest.raises(ValueError, match=msg):
        hexio.read_hex(p, 3 if msg.startswith("2 words") else 2)
    with pytest.raises(FileNotFoundError):
        hexio.read_hex(tmp_path / "missing.hex", 1)


def test_load_real_npy_checks(tmp_path, fs):
    good = _f32(fs["v"])
    p = tmp_path / "v.npy"
    np.save(p, good)
    assert np.array_equal(hexio.load_real_npy(p, (1, 128, 128)), good)
    with pytest.raises(hexio.VectorFileError, match=r"shape \(1, 128, 128\), want \(4, 128, 128\)"):
        hexio.load_real_npy(p, (4, 128, 128))
    np.save(p, good.astype(np.float64))
    with pytest.raises(hexio.VectorFileError, match="dtype float64, want float32"):
        hexio.load_real_npy(p, (1, 128, 128))
    bad = good.copy()
    bad[0, 0, 0] = np.nan
    bad[0, 0, 1] = np.float32(1.0000001)
    bad[0, 0, 2] = np.float32(1.0000001)
    np.save(p, bad)
    # every problem is reported in one error
    with pytest.raises(hexio.VectorFileError, match="1 NaN/Inf words; 2 words that are not bf16"):
        hexio.load_real_npy(p, (1, 128, 128))
    np.save(p, bad[:, :64])
    with pytest.raises(hexio.VectorFileError, match="shape .*; 1 NaN/Inf words; 2 words"):
        hexio.load_real_npy(p, (1, 128, 128))
    p.write_bytes(b"version https://git-lfs.github.com/spec/v1\noid sha256:00\nsize 1\n")
    with pytest.raises(hexio.VectorFileError, match="Git LFS placeholder"):
        hexio.load_real_npy(p, (1, 128, 128))
    with pytest.raises(FileNotFoundError):
        hexio.load_real_npy(tmp_path / "missing.npy", (1, 128, 128))


def test_prepare_from_npy_and_existing_check(tmp_path, fs, sha):
    gdir = tmp_path / "golden_model_outputs" / "fpga_slice"
    gdir.mkdir(parents=True)
    for name in hexio.SHAPES:
        np.save(gdir / name, _f32(fs[name[:-4]]))
    out = tmp_path / "tb"
    man = hexio.prepare_from_npy(gdir, out)
    for name, entry in man["outputs"].items():
        assert entry["sha256"] == sha[name]
    assert set(man["sources"]) == set(hexio.SHAPES)
    # an existing file that disagrees is reported with the first differing word
    wrong = fs["softmax_weights"].copy()
    wrong.reshape(-1)[77] ^= 1
    ex = tmp_path / "existing.hex"
    hexio.write_hex(ex, wrong)
    with pytest.raises(RuntimeError, match="1 of 65536 words differ .* first at word 77"):
        hexio.prepare_from_npy(gdir, tmp_path / "tb2", existing={"softmax_weights.npy": ex})
