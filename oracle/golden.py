"""ctypes wrapper over gqa_oracle.c -- TEST INFRASTRUCTURE ONLY.

Restates the bf16-staged golden model (reference file
llama3_attention_golden_model.py) on bf16 words held in ``np.uint16`` arrays:

=====================  ==============================================
function               reference it follows
=====================  ==============================================
``to_bf16_words``      ``to_bf16`` :44-47
``rope_table``         ``build_rope_cache`` :124-130
``rope_apply``         ``rotate_half`` / ``apply_rope`` :133-139, :162-164
``scores``             ``to_bf16(matmul(q, k^T) * scale)`` :175-176
``mask_golden``        ``to_bf16(scores + triu(-inf))`` :180-181
``attention_mask``     HLS ``attention_mask`` attention_mask_module/src/attention_mask.cpp:3-58
``softmax``            ``to_bf16(F.softmax(...))`` :185
``pv``                 ``to_bf16(matmul(weights, v))`` :189
``stages``             ``run_full_attention`` :157-190 (core part)
``attention_rows``     exact (float64) attention on sampled rows
=====================  ==============================================
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libgqa_oracle.so")
_lib = None

ROPE_THETA = 500000.0
MASK_NEG_INF_BF16 = 0xFF80


def build() -> str:
    """Compile the oracle shared library with make (gcc)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    src = os.path.join(_HERE, "gqa_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
    f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
    i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
    ci, cl, cf, cd = ctypes.c_int, ctypes.c_long, ctypes.c_float, ctypes.c_double
    lib.orc_f32_to_bf16_array.argtypes = [f32p, u16p, cl]
    lib.orc_bf16_to_f32_array.argtypes = [u16p, f32p, cl]
    lib.orc_inv_freq.argtypes = [ci, cd, f32p]
    lib.orc_rope_table.argtypes = [ci, ci, ci, cd, u16p, u16p]
    lib.orc_rope_apply.argtypes = [u16p, u16p, u16p, u16p, ci, ci, ci]
    lib.orc_scores.argtypes = [u16p, u16p, u16p, ci, ci, ci, ci, cf]
    lib.orc_mask_golden.argtypes = [u16p, u16p, ci, ci, ci]
    lib.orc_attention_mask_words.argtypes = [u16p, u16p, ci, ci, ci, ctypes.c_uint16]
    lib.orc_attention_mask_words.restype = ci
    lib.orc_softmax.argtypes = [u16p, u16p, cl, ci]
    lib.orc_pv.argtypes = [u16p, u16p, u16p, ci, ci, ci, ci]
    lib.orc_attention_rows.argtypes = [u16p, u16p, u16p, ci, ci, ci, ci, ci, cf, ci, i32p, i32p,
                                       ctypes.c_void_p, ci, f32p]
    lib.orc_set_num_threads.argtypes = [ci]
    lib.orc_num_threads.restype = ci
    _lib = lib
    return lib


def set_num_threads(n: int) -> None:
    _load().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(_load().orc_num_threads())


def _u16(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.uint16)


def to_bf16_words(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 words, round to nearest even (golden ``to_bf16`` :44-47)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    _load().orc_f32_to_bf16_array(x.reshape(-1), out.reshape(-1), x.size)
    return out


def bf16_words_to_f32(w: np.ndarray) -> np.ndarray:
    """bf16 words -> exact fp32 values."""
    return (_u16(w).astype(np.uint32) << 16).view(np.float32)


def scale_for(head_dim: int) -> float:
    """fl32(1/sqrt(d)) as the golden's ``tensor * python_float`` uses it (:175)."""
    return float(np.float32(1.0 / math.sqrt(head_dim)))


def inv_freq(head_dim: int = 128, theta: float = ROPE_THETA) -> np.ndarray:
    out = np.empty(head_dim // 2, np.float32)
    _load().orc_inv_freq(head_dim, float(theta), out)
    return out


def rope_table(seq_len: int, head_dim: int = 128, theta: float = ROPE_THETA, pos0: int = 0):
    """(cos, sin) bf16 words [S][D] (golden ``build_rope_cache`` :124-130)."""
    c = np.empty((seq_len, head_dim), np.uint16)
    s = np.empty((seq_len, head_dim), np.uint16)
    _load().orc_rope_table(seq_len, pos0, head_dim, float(theta), c, s)
    return c, s


def rope_apply(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """bf16(x*cos + rotate_half(x)*sin) for x [H][S][D] (golden :133-139)."""
    x = _u16(x)
    H, S, D = x.shape
    y = np.empty_like(x)
    _load().orc_rope_apply(x, y, _u16(cos[:S]), _u16(sin[:S]), H, S, D)
    return y


def scores(q: np.ndarray, k: np.ndarray, scale: float | None = None) -> np.ndarray:
    """bf16(fl32(q.k) * scale) for q [Hq][S][D], k [Hkv][S][D] (golden :175-176)."""
    q, k = _u16(q), _u16(k)
    Hq, S, D = q.shape
    Hkv = k.shape[0]
    out = np.empty((Hq, S, S), np.uint16)
    _load().orc_scores(q, k, out, Hq, Hkv, S, D, scale_for(D) if scale is None else float(scale))
    return out


def mask_golden(s: np.ndarray, causal: bool = True) -> np.ndarray:
    """bf16(scores + triu(-inf, 1)) (golden :180-181)."""
    s = _u16(s)
    H, S, _ = s.shape
    out = np.empty_like(s)
    _load().orc_mask_golden(s, out, H, S, int(causal))
    return out


def attention_mask(raw: np.ndarray, q_heads: int, seq_len: int, causal: bool = True,
                   mask_value: int = MASK_NEG_INF_BF16) -> np.ndarray:
    """Word pass-through mask of the HLS kernel (attention_mask.cpp:3-58)."""
    raw = _u16(raw).reshape(-1)
    out = np.empty_like(raw)
    rc = _load().orc_attention_mask_words(raw, out, q_heads, seq_len, int(causal), mask_value)
    if rc != 0:
        raise ValueError("invalid attention_mask sizes")
    return out


def softmax(s: np.ndarray) -> np.ndarray:
    """bf16(softmax(s, -1)) over bf16 words (golden :185)."""
    s = _u16(s)
    out = np.empty_like(s)
    cols = s.shape[-1]
    _load().orc_softmax(s.reshape(-1, cols), out.reshape(-1, cols), s.size // cols, cols)
    return out


def pv(p: np.ndarray, v: np.ndarray) -> np.ndarray:
    """bf16(sum_j p*v) with fp32 j-order accumulation (golden :189)."""
    p, v = _u16(p), _u16(v)
    Hq, S, _ = p.shape
    Hkv, _, D = v.shape
    out = np.empty((Hq, S, D), np.uint16)
    _load().orc_pv(p, v, out, Hq, Hkv, S, D)
    return out


def stages(q_raw: np.ndarray, k_raw: np.ndarray, v: np.ndarray, causal: bool = True,
           theta: float = ROPE_THETA) -> dict:
    """Every golden stage of the attention core for one batch element.

    q_raw [Hq][S][D], k_raw/v [Hkv][S][D] bf16 words (pre-RoPE), returns a dict
    keyed by the golden model's dump names (llama3_attention_golden_model.py:157-190).
    """
    q_raw, k_raw, v = _u16(q_raw), _u16(k_raw), _u16(v)
    S, D = q_raw.shape[1], q_raw.shape[2]
    cos, sin = rope_table(S, D, theta)
    qr = rope_apply(q_raw, cos, sin)
    kr = rope_apply(k_raw, cos, sin)
    sc = scores(qr, kr)
    sm = mask_golden(sc, causal)
    w = softmax(sm)
    out = pv(w, v)
    return {
        "q_before_rope": q_raw, "k_before_rope": k_raw, "v": v,
        "cos": cos, "sin": sin,
        "q_after_rope": qr, "k_after_rope": kr,
        "scores_before_mask": sc, "scores_after_mask": sm,
        "softmax_weights": w, "attn_out_per_head": out,
    }


def attention_rows(q: np.ndarray, k: np.ndarray, v: np.ndarray, row_head, row_pos, causal: bool = True,
                   n_keys=None, scale: float | None = None) -> np.ndarray:
    """Exact (float64-accumulated) attention outputs for selected (head, position) rows.

    q [Hq][Sq][D] and k [Hkv][Sk][D] already rotated; returns fp32 [n][D].
    """
    q, k, v = _u16(q), _u16(k), _u16(v)
    Hq, Sq, D = q.shape
    Hkv, Sk, _ = k.shape
    rh = np.ascontiguousarray(row_head, np.int32)
    rp = np.ascontiguousarray(row_pos, np.int32)
    nk = None if n_keys is None else np.ascontiguousarray(n_keys, np.int32)
    out = np.empty((rh.size, D), np.float32)
    _load().orc_attention_rows(q, k, v, Hq, Hkv, Sq, Sk, D, scale_for(D) if scale is None else float(scale),
                               int(causal), rh, rp, None if nk is None else nk.ctypes.data, rh.size, out)
    return out


def read_hex_words(path: str, bits: int = 16) -> np.ndarray:
    """One hex word per line (LF or CRLF) -> uint16 (bits=16) or uint32 (bits=32) array."""
    with open(path, "r", encoding="ascii") as f:
        vals = [int(t, 16) for t in f.read().split()]
    return np.asarray(vals, dtype=np.uint16 if bits == 16 else np.uint32)
