"""Regenerate the golden fixtures under tests/golden/ from the reference repository.

Run where a checkout of the reference repository is available (read-only is fine):

    python tests/golden/make_fixtures.py --reference <path to the reference checkout>

(or set GQA_REFERENCE_DIR instead of passing --reference).

Writes:

* ``fpga_slice.npz`` -- the reference's committed hex golden vectors for its
  fpga_slice (KV group 0: 4 Q heads x 1 KV head x 128 tokens x 128 dims), as
  bf16 words (uint16).  Sources (paths inside the reference):
    A_attention_integration_final_v5/tb/golden_fpga_slice_data/*.hex
    attention_mask_module/mask_test_vectors/{raw_scores,golden_masked_scores}.hex
    FPT_BC_QK_Softmax_PV_Delivery_v5/data/full_qk_optional/scores_before_mask.hex
    softmax_module/data/{input_scores_bf16,expected_probs_bf16,input_masks}.mem
  The SHA-256 of every hex file is checked against
  golden_fpga_slice_data/attention_fpga_slice_manifest.json where listed.

* ``fpga_slice_sha256.json`` -- the SHA-256 that the reference's manifest lists for
  each of those hex files (upper-case hex convention), so emitted hex files can be
  checked byte for byte.

* ``layer_s32.npz`` -- every stage dump of the reference's own
  ``run_full_attention`` (llama3_attention_golden_model.py:144-197), imported
  and run here on seeded synthetic inputs: hidden [32, 4096] ~ N(0,1) and
  Wq [4096,4096], Wk/Wv [1024,4096], Wo [4096,4096] ~ N(0, 0.02^2), all drawn
  with numpy default_rng(LAYER_SEED) in that order and rounded to bf16.  The
  weights are not stored; ``layer_inputs()`` regenerates them bit-identically.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LAYER_SEED = 20260
LAYER_SEQ = 32
HIDDEN = 4096


def _hex(path: str, bits: int = 16) -> np.ndarray:
    with open(path, "r", encoding="ascii") as f:
        vals = [int(t, 16) for t in f.read().split()]
    return np.asarray(vals, dtype=np.uint16 if bits == 16 else np.uint32)


def _sha(path: str) -> str:
    """SHA-256 of the file with hex digits upper-cased (the manifest's convention;
    three of the committed files were re-written in lower case with equal values)."""
    with open(path, "rb") as f:
        return hashlib.sha256(f.read().upper()).hexdigest()


def bf16_round_np(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 words (RNE)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def layer_inputs(seed: int = LAYER_SEED, seq: int = LAYER_SEQ):
    """(hidden, wq, wk, wv, wo) as bf16 words, drawn exactly as the fixture was."""
    rng = np.random.default_rng(seed)
    h = bf16_round_np(rng.standard_normal((seq, HIDDEN), dtype=np.float32))
    wq = bf16_round_np(rng.standard_normal((HIDDEN, HIDDEN), dtype=np.float32) * np.float32(0.02))
    wk = bf16_round_np(rng.standard_normal((1024, HIDDEN), dtype=np.float32) * np.float32(0.02))
    wv = bf16_round_np(rng.standard_normal((1024, HIDDEN), dtype=np.float32) * np.float32(0.02))
    wo = bf16_round_np(rng.standard_normal((HIDDEN, HIDDEN), dtype=np.float32) * np.float32(0.02))
    return h, wq, wk, wv, wo


def make_fpga_slice(ref: str) -> dict:
    gd = os.path.join(ref, "A_attention_integration_final_v5/tb/golden_fpga_slice_data")
    with open(os.path.join(gd, "attention_fpga_slice_manifest.json")) as f:
        manifest = json.load(f)["outputs"]
    files = {
        "q_before_rope": ("q_before_rope_bf16.hex", (4, 128, 128)),
        "k_before_rope": ("k_before_rope_bf16.hex", (1, 128, 128)),
        "v": ("v_bf16.hex", (1, 128, 128)),
        "q_after_rope": ("q_after_rope_golden_bf16.hex", (4, 128, 128)),
        "k_after_rope": ("k_after_rope_golden_bf16.hex", (1, 128, 128)),
        "softmax_weights": ("softmax_weights_bf16.hex", (4, 128, 128)),
        "attn_out_per_head": ("attn_out_per_head_bf16.hex", (4, 128, 128)),
        "sin_pairs": ("sin_bf16.hex", (128, 64)),
        "cos_pairs": ("cos_bf16.hex", (128, 64)),
    }
    out = {}
    for key, (fname, shape) in files.items():
        path = os.path.join(gd, fname)
        want = manifest.get(fname, {}).get("sha256")
        if want is not None and _sha(path) != want:
            raise SystemExit(f"sha256 mismatch for {path}")
        out[key] = _hex(path).reshape(shape)
    extra = {
        "scores_before_mask": ("FPT_BC_QK_Softmax_PV_Delivery_v5/data/full_qk_optional/scores_before_mask.hex", 16),
        "mask_raw_scores": ("attention_mask_module/mask_test_vectors/raw_scores.hex", 16),
        "scores_after_mask": ("attention_mask_module/mask_test_vectors/golden_masked_scores.hex", 16),
        "softmax_input_scores": ("softmax_module/data/input_scores_bf16.mem", 16),
        "softmax_expected_probs": ("softmax_module/data/expected_probs_bf16.mem", 16),
        "softmax_input_masks": ("softmax_module/data/input_masks.mem", 16),
        "pv_softmax_weights": ("PV_module/sim_data/softmax_weights_bf16.hex", 16),
        "pv_v": ("PV_module/sim_data/v_bf16.hex", 16),
        "pv_attn_out": ("PV_module/sim_data/attn_out_per_head_bf16.hex", 16),
        "rope_q_after": ("RoPE/data/q_after_rope_golden_bf16.hex", 16),
        "rope_k_after": ("RoPE/data/k_after_rope_golden_bf16.hex", 16),
    }
    for key, (rel, bits) in extra.items():
        arr = _hex(os.path.join(ref, rel), bits)
        n = arr.size
        out[key] = arr.reshape((4, 128, 128) if n == 65536 else (1, 128, 128) if n == 16384 else (n,))
    return out


def slice_sha256(ref: str) -> dict:
    """Manifest SHA-256 of each slice hex file, plus a digest of the full 8192-token RoPE
    ROM words (``rom_<sin|cos>_words``: SHA-256 of the little-endian uint16 words of
    RoPE/<sin|cos>_bf16_all.hex, which has CRLF line ends)."""
    gd = os.path.join(ref, "A_attention_integration_final_v5/tb/golden_fpga_slice_data")
    with open(os.path.join(gd, "attention_fpga_slice_manifest.json")) as f:
        manifest = json.load(f)["outputs"]
    out = {name: entry["sha256"] for name, entry in sorted(manifest.items()) if "sha256" in entry}
    for name in ("sin", "cos"):
        words = _hex(os.path.join(ref, "RoPE", f"{name}_bf16_all.hex"))
        out[f"rom_{name}_words"] = hashlib.sha256(words.astype("<u2").tobytes()).hexdigest()
    return out


def _import_golden(ref: str):
    spec = importlib.util.spec_from_file_location(
        "llama3_attention_golden_model", os.path.join(ref, "llama3_attention_golden_model.py"))
    mod = importlib.util.module_from_spec(spec)
    cwd = os.getcwd()
    with tempfile.TemporaryDirectory() as tmp:
        os.chdir(tmp)  # the module creates ./golden_model_outputs on import
        try:
            spec.loader.exec_module(mod)
        finally:
            os.chdir(cwd)
    return mod


def make_layer(ref: str) -> dict:
    import torch

    gm = _import_golden(ref)
    h, wq, wk, wv, wo = layer_inputs()

    def t(w):
        return torch.from_numpy((w.astype(np.uint32) << 16).view(np.float32).copy())

    dump = gm.run_full_attention(t(h), t(wq), t(wk), t(wv), t(wo))
    out = {}
    for key, ten in dump.items():
        out[key] = bf16_round_np(ten.detach().float().contiguous().numpy())
    out["hidden_states_input"] = h
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("GQA_REFERENCE_DIR"),
                    help="path of the reference checkout (default: $GQA_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference or GQA_REFERENCE_DIR")
    fs = make_fpga_slice(args.reference)
    np.savez_compressed(os.path.join(HERE, "fpga_slice.npz"), **fs)
    with open(os.path.join(HERE, "fpga_slice_sha256.json"), "w") as f:
        json.dump(slice_sha256(args.reference), f, indent=1)
        f.write("\n")
    layer = make_layer(args.reference)
    np.savez_compressed(os.path.join(HERE, "layer_s32.npz"), **layer)
    for name in ("fpga_slice.npz", "layer_s32.npz"):
        p = os.path.join(HERE, name)
        print(name, os.path.getsize(p), "bytes")


if __name__ == "__main__":
    sys.exit(main())
