"""BF16 hex fixture I/O: the reference's RTL test-bench vector format, produced from GPU
stage dumps.

The reference turns its golden-model dumps into one-word-per-line hex files for the
Verilog test benches (A_attention_integration_final_v5/scripts/
prepare_attention_fpga_slice_vectors.py).  This module writes the same files, with the
same names, word order and format, from this package's GPU stage kernels.  The file
format, names and manifest fields are the reference's (the test benches read them); the
readers and checks are this module's own, and raise VectorFileError (a ValueError):

=============================  ====================================================
function                       reference (prepare_attention_fpga_slice_vectors.py)
=============================  ====================================================
``SHAPES``, ``NPY_TO_HEX``     :20-38 (slice shapes and file names)
``load_real_npy``              :49-72 (the same checks: LFS pointer, shape, dtype, finite, bf16)
``bf16_words``                 :75-77
``read_hex``                   :80-97 (the same format: blank lines skipped, 16-bit words,
                               exact count)
``write_hex``                  :100-103 (``%04X`` + LF)
``assert_existing_hex_matches`` :106-119 (same purpose)
``emit_fpga_slice``            :171-249 (hex files, sin/cos tables, manifest)
=============================  ====================================================

``rope_rom_words`` builds the RoPE sin/cos ROM tables ``[token][pair]`` that the test
benches read (RoPE/tools/prepare_rope_vectors.py copies them from the 8192-entry ROM
``RoPE/{sin,cos}_bf16_all.hex``): float64 angles and sin/cos, rounded to fp32 and then
to bf16.  These are the RTL's tables, which differ from the golden model's fp32-angle
cache in a few entries; the GPU RoPE kernel follows the golden model.

``fpga_slice_from_hex`` is the end-to-end GPU flow: read the slice's input hex files
(q/k before RoPE, v), run every attention stage on the GPU, and write all the golden
hex files a test bench compares against.
"""
from __future__ import annotations

import hashlib
import json
import re
from pathlib import Path

import numpy as np
import torch

SHAPES = {
    "q_before_rope.npy": (4, 128, 128),
    "k_before_rope.npy": (1, 128, 128),
    "v.npy": (1, 128, 128),
    "q_after_rope.npy": (4, 128, 128),
    "k_after_rope.npy": (1, 128, 128),
    "softmax_weights.npy": (4, 128, 128),
    "attn_out_per_head.npy": (4, 128, 128),
}

NPY_TO_HEX = {
    "q_before_rope.npy": "q_before_rope_bf16.hex",
    "k_before_rope.npy": "k_before_rope_bf16.hex",
    "v.npy": "v_bf16.hex",
    "q_after_rope.npy": "q_after_rope_golden_bf16.hex",
    "k_after_rope.npy": "k_after_rope_golden_bf16.hex",
    "softmax_weights.npy": "softmax_weights_bf16.hex",
    "attn_out_per_head.npy": "attn_out_per_head_bf16.hex",
}

ROM_TABLES = ("sin_bf16.hex", "cos_bf16.hex")

MANIFEST_NAME = "attention_fpga_slice_manifest.json"


class VectorFileError(ValueError):
    """A golden tensor or hex vector file that the test benches cannot use."""


def sha256(path) -> str:
    """Hex SHA-256 digest of a file (the manifest's checksum; vector files are small)."""
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


_LFS_SIGNATURE = b"version https://git-lfs.github.com/spec/v1"


def load_real_npy(path, shape: tuple) -> np.ndarray:
    """Load one golden tensor: float32 storage holding bf16 values of the given shape.

    Every problem found is reported at once in one VectorFileError: a Git LFS placeholder
    instead of the array, a shape or dtype other than expected, and (on float32 data)
    the number of NaN/Inf words and of words whose low 16 bits are set (values a bf16
    word cannot hold).  The checks on the words are one pass over their bit patterns."""
    path = Path(path)
    with path.open("rb") as fh:  # FileNotFoundError for a missing tensor
        if fh.read(len(_LFS_SIGNATURE)) == _LFS_SIGNATURE:
            raise VectorFileError(f"{path}: Git LFS placeholder; fetch the LFS object before converting")
    arr = np.load(path, allow_pickle=False)
    problems = []
    if arr.shape != tuple(shape):
        problems.append(f"shape {arr.shape}, want {tuple(shape)}")
    if arr.dtype != np.float32:
        problems.append(f"dtype {arr.dtype}, want float32")
    else:
        bits = np.ascontiguousarray(arr).view(np.uint32)
        n_nonfinite = int(np.count_nonzero((bits & 0x7F800000) == 0x7F800000))
        n_wide = int(np.count_nonzero(bits & 0xFFFF))
        if n_nonfinite:
            problems.append(f"{n_nonfinite} NaN/Inf words")
        if n_wide:
            problems.append(f"{n_wide} words that are not bf16 (low 16 bits set)")
    if problems:
        raise VectorFileError(f"{path.name}: " + "; ".join(problems))
    return arr


def bf16_words(x) -> np.ndarray:
    """bf16 words (uint16) of a bf16 tensor, or of bf16-exact values in fp32 storage
    (a tensor or an array; values that are not bf16-exact raise)."""
    if isinstance(x, torch.Tensor):
        t = x.detach().cpu()
        if t.dtype == torch.bfloat16:
            return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
        x = t.to(torch.float32).numpy()
    a = np.ascontiguousarray(x, dtype=np.float32)
    bits = a.view(np.uint32)
    if np.any(bits & np.uint32(0xFFFF)):
        raise ValueError("values are not exact BF16 values")
    return (bits >> np.uint32(16)).astype(np.uint16)


_HEX_WORD = re.compile(r"0*[0-9A-Fa-f]{1,4}")  # a 16-bit word (leading zeros allowed)


def read_hex(path, expected_words: int) -> np.ndarray:
    """Parse a hex vector file: one 16-bit word per non-blank line (CR/LF, any case).

    A missing file raises FileNotFoundError; a line that is not a 16-bit hex word, or a
    word count other than `expected_words`, raises VectorFileError naming the file (and
    the first offending line)."""
    path = Path(path)
    text = path.read_text(encoding="ascii")
    lines = [(no, ln.strip()) for no, ln in enumerate(text.splitlines(), 1)]
    tokens = [(no, tok) for no, tok in lines if tok]
    for no, tok in tokens:
        if not _HEX_WORD.fullmatch(tok):
            raise VectorFileError(f"{path}, line {no}: {tok!r} is not a 16-bit hex word")
    if len(tokens) != expected_words:
        raise VectorFileError(f"{path}: {len(tokens)} words, want {expected_words}")
    return np.array([int(tok, 16) for _, tok in tokens], dtype=np.uint16)


def write_hex(path, words) -> None:
    """Upper-case 4-digit words, one per line, LF endings, C-order flattening."""
    flat = np.asarray(words, dtype=np.uint16).reshape(-1)
    text = "".join(f"{int(w):04X}\n" for w in flat)
    with open(path, "w", encoding="ascii", newline="\n") as handle:
        handle.write(text)


def assert_existing_hex_matches(existing, generated, logical_name: str) -> None:
    """When `existing` names a file, it must hold exactly the `generated` words;
    otherwise RuntimeError reports how many words differ and where the first one is."""
    existing = Path(existing)
    if not existing.is_file():
        return
    gen = np.asarray(generated, dtype=np.uint16).ravel()
    old = read_hex(existing, gen.size)
    diff = old != gen
    if diff.any():
        first = int(diff.argmax())
        raise RuntimeError(f"{logical_name}: {int(diff.sum())} of {gen.size} words differ from {existing}, "
                           f"first at word {first} (now {gen[first]:04X}, file has {old[first]:04X})")


def _bf16_rne(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 words, round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def rope_rom_words(seq_len: int = 128, head_dim: int = 128, theta: float = 500000.0, pos0: int = 0):
    """RoPE ROM tables (sin, cos) as bf16 words [seq_len][head_dim // 2]: angle =
    pos / theta^(2i/d), angle and sin/cos in float64, rounded to fp32 and then to bf16
    (round to nearest even both times), for pos in [pos0, pos0 + seq_len).  This
    reproduces the reference's 8192-entry ROM word for word."""
    i = np.arange(0, head_dim, 2, dtype=np.float64)
    inv = 1.0 / (theta ** (i / head_dim))
    ang = np.outer(np.arange(pos0, pos0 + seq_len, dtype=np.float64), inv)
    return _bf16_rne(np.sin(ang).astype(np.float32)), _bf16_rne(np.cos(ang).astype(np.float32))


def emit_fpga_slice(arrays: dict, out_dir, *, existing: dict | None = None, sources: dict | None = None,
                    seq_len: int = 128, theta: float = 500000.0, kv_groups: int = 8) -> dict:
    """Write the slice's hex files, the RoPE ROM tables and the manifest into `out_dir`.

    `arrays` maps the .npy names of ``SHAPES`` (or their stems) to tensors / arrays of
    bf16 values with those shapes.  `existing` optionally maps the same names to hex
    files that must already hold the same words.  Returns the manifest dict."""
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    outputs = {}
    for npy_name, hex_name in NPY_TO_HEX.items():
        stem = npy_name[:-4]
        src = arrays[npy_name] if npy_name in arrays else arrays[stem]
        words = bf16_words(src)
        if words.shape != SHAPES[npy_name]:
            raise ValueError(f"{npy_name}: expected shape {SHAPES[npy_name]}, got {words.shape}")
        if existing and (npy_name in existing or stem in existing):
            assert_existing_hex_matches(existing.get(npy_name, existing.get(stem)), words, npy_name)
        path = out_dir / hex_name
        write_hex(path, words)
        outputs[hex_name] = {"words": int(words.size), "sha256": sha256(path), "source": npy_name}
    sin_w, cos_w = rope_rom_words(seq_len, 128, theta)
    for hex_name, words in zip(ROM_TABLES, (sin_w, cos_w)):
        path = out_dir / hex_name
        write_hex(path, words)
        outputs[hex_name] = {"words": int(words.size), "sha256": sha256(path),
                             "source": f"float64-angle RoPE ROM, tokens 0..{seq_len - 1}"}
    manifest = {
        "purpose": "Raw Q/K -> RoPE -> QK -> causal mask -> Softmax -> real PV -> Context",
        "configuration": {
            "physical_gqa_groups": kv_groups,
            "run_gqa_groups": 1,
            "q_heads_per_group": 4,
            "seq_len": seq_len,
            "head_dim": 128,
            "rope_pairing": "x0=dimension[pair], x1=dimension[pair+64]",
        },
        "sources": sources or {},
        "outputs": outputs,
    }
    (out_dir / MANIFEST_NAME).write_text(json.dumps(manifest, indent=2) + "\n", encoding="utf-8")
    return manifest


def prepare_from_npy(golden_dir, out_dir, *, existing: dict | None = None) -> dict:
    """The reference's flow: validate golden_model_outputs/fpga_slice/*.npy (as written by
    ``golden_model.save_dump``) and emit the hex files and manifest."""
    golden_dir = Path(golden_dir)
    arrays, sources = {}, {}
    for name, shape in SHAPES.items():
        path = golden_dir / name
        arrays[name] = load_real_npy(path, shape)
        sources[name] = {"path": path.name, "shape": list(shape), "dtype": "float32", "sha256": sha256(path)}
    return emit_fpga_slice(arrays, out_dir, existing=existing, sources=sources)


def fpga_slice_from_hex(in_dir, out_dir, *, device=None, existing: bool = False) -> dict:
    """Read q/k before RoPE and v from `in_dir`'s hex files, run every stage on the GPU
    (bit-exact stage kernels), and write the full set of slice hex files to `out_dir`.
    With `existing=True` every output that also exists in `in_dir` must match it."""
    from . import golden_model

    in_dir = Path(in_dir)
    words = {}
    for npy_name in ("q_before_rope.npy", "k_before_rope.npy", "v.npy"):
        shape = SHAPES[npy_name]
        words[npy_name] = read_hex(in_dir / NPY_TO_HEX[npy_name], int(np.prod(shape))).reshape(shape)

    def as_f32(w):
        return torch.from_numpy((w.astype(np.uint32) << np.uint32(16)).view(np.float32).copy())

    dev = torch.device(device) if device is not None else None
    q, k, v = (as_f32(words[n]) for n in ("q_before_rope.npy", "k_before_rope.npy", "v.npy"))
    if dev is not None:
        q, k, v = q.to(dev), k.to(dev), v.to(dev)
    dump = golden_model.run_attention_core(q, k, v, debug=True)
    arrays = {name: dump[name[:-4]] for name in SHAPES}
    sources = {n: {"path": NPY_TO_HEX[n], "sha256": sha256(in_dir / NPY_TO_HEX[n])} for n in words}
    ex = {n: in_dir / h for n, h in NPY_TO_HEX.items()} if existing else None
    return emit_fpga_slice(arrays, out_dir, existing=ex, sources=sources)
