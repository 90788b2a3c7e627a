"""ctypes binding of libgqa_b200.so (the C ABI declared in include/gqa_b200.h).

The library is required: if it is missing or fails to load, every entry point
raises -- there is no CPU or PyTorch fallback for the kernels.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgqa_b200.so")

GQA_OK = 0
GQA_ERR_INVALID_ARGUMENT = -1
GQA_ERR_UNSUPPORTED = -2
GQA_ERR_MISALIGNED = -3
GQA_ERR_CUDA = -4
GQA_ERR_DEVICE_TIMEOUT = -5
GQA_ERR_WORKSPACE = -6
GQA_ERR_NO_DEVICE = -7
GQA_ERR_DEVICE_INPUT = -8

GQA_FLAG_CAUSAL = 1
GQA_FLAG_ROPE_Q = 2
GQA_FLAG_ROPE_K = 4
GQA_MASK_NEG_INF_BF16 = 0xFF80
GQA_GEMM_OUT_F32 = 1

# (name, restype, argtypes) for every symbol include/gqa_b200.h declares.
_vp, _i, _f, _d, _ll, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double, ctypes.c_longlong, ctypes.c_size_t
SIGNATURES = {
    "gqa_strerror": (ctypes.c_char_p, [_i]),
    "gqa_version": (_i, []),
    "gqa_device_check": (_i, [_vp, ctypes.POINTER(_i)]),
    "gqa_rope_cache_bf16": (_i, [_vp, _vp, _i, _i, _i, _d, _vp]),
    "gqa_rope_bf16": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "gqa_scores_bf16": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp]),
    "gqa_mask_bf16": (_i, [_vp, _vp, _i, _i, _i, _vp]),
    "gqa_attention_mask_bf16": (_i, [_vp, _vp, _i, _i, _i, ctypes.c_uint16, _vp]),
    "gqa_softmax_bf16": (_i, [_vp, _vp, _ll, _i, _vp]),
    "gqa_pv_bf16": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "gqa_prefill_bf16": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _i, _vp]),
    "gqa_decode_workspace_size": (_sz, [_i, _i, _i, _i]),
    "gqa_decode_bf16": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i, _i, _i, _i, _i, _i, _i, _i, _f,
                             _i, _vp]),
    "gqa_decode_noalloc_scratch_bytes": (_sz, []),
    "gqa_decode_bf16_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _f, _i,
                                     _vp]),
    "gqa_kv_append_bf16": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i,
                                _vp]),
    "gqa_decode_paged_bf16": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i, _i, _i, _i,
                                   _i, _i, _i, _f, _i, _vp]),
    "gqa_gemm_bf16": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "gqa_qkv_proj_bf16": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "gqa_o_proj_bf16": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "gqa_cast_f32_bf16": (_i, [_vp, _vp, _ll, _vp]),
    "gqa_tp_buffer_bytes": (_sz, [_i, _i]),
    "gqa_peer_handle_bytes": (_sz, []),
    "gqa_peer_alloc": (_i, [_sz, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]),
    "gqa_peer_open": (_i, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "gqa_peer_close": (_i, [_vp]),
    "gqa_peer_free": (_i, [_vp]),
    "gqa_tp_reduce_gather_bf16": (_i, [ctypes.POINTER(ctypes.c_void_p), _i, _i, _i, _i, ctypes.c_uint, _vp]),
    "gqa_tp_o_proj_exchange_bf16": (_i, [_vp, _vp, _i, ctypes.POINTER(ctypes.c_void_p), _i, _i, _i, _i, _i, _i,
                                         ctypes.c_uint, _vp]),
    "gqa_o_proj_rows_bf16": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
}


class GqaError(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what}: {strerror(code)} ({code})")


_lib = None
_lock = threading.Lock()


def load(build_if_missing: bool = False):
    """Load (once) and return the ctypes handle; raises if the library is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            if build_if_missing:
                from . import build as _build
                _build.build()
            else:
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m llama3_8b_attention_optimize_b200.build` "
                    "(the CUDA kernels have no fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def strerror(code: int) -> str:
    try:
        return load().gqa_strerror(code).decode()
    except Exception:  # pragma: no cover - used while reporting another error
        return "unknown"


def check(code: int, what: str) -> None:
    if code != GQA_OK:
        raise GqaError(code, what)


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
