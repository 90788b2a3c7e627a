"""C-ABI checks that need no GPU: the library loads, exports every declared
symbol, and rejects bad arguments on the host before touching a device."""
import ctypes
import os
import re

import pytest

from llama3_8b_attention_optimize_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    with open(os.path.join(ROOT, "include", "gqa_b200.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(gqa_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return _lib.load(build_if_missing=True)


def test_every_declared_symbol_is_exported(lib):
    declared = _declared_symbols()
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(_lib.exported_symbols()) == declared


def test_version_and_strerror(lib):
    assert lib.gqa_version() >= 10000
    for code in range(0, -8, -1):
        assert lib.gqa_strerror(code)
    assert b"unknown" in lib.gqa_strerror(-99)


def test_host_validation_rejects_bad_arguments(lib):
    E = _lib
    # null pointers
    assert lib.gqa_prefill_bf16(None, None, None, None, None, None, 1, 128, 32, 8, 128, 0, 8, 0.088, 1, None) == \
        E.GQA_ERR_INVALID_ARGUMENT
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: validation fails first
    mis = ctypes.c_void_p(0x1002)
    # unsupported head_dim / group size
    assert lib.gqa_prefill_bf16(fake, fake, fake, fake, None, None, 1, 128, 32, 8, 64, 0, 8, 0.1, 1, None) == \
        E.GQA_ERR_UNSUPPORTED
    assert lib.gqa_prefill_bf16(fake, fake, fake, fake, None, None, 1, 128, 32, 16, 128, 0, 16, 0.1, 1, None) == \
        E.GQA_ERR_UNSUPPORTED
    # bad kv-head range, bad flags, rope without tables, bad scale
    assert lib.gqa_prefill_bf16(fake, fake, fake, fake, None, None, 1, 128, 32, 8, 128, 6, 4, 0.1, 1, None) == \
        E.GQA_ERR_INVALID_ARGUMENT
    assert lib.gqa_prefill_bf16(fake, fake, fake, fake, None, None, 1, 128, 32, 8, 128, 0, 8, 0.1, 64, None) == \
        E.GQA_ERR_INVALID_ARGUMENT
    assert lib.gqa_prefill_bf16(fake, fake, fake, fake, None, None, 1, 128, 32, 8, 128, 0, 8, 0.1, 2, None) == \
        E.GQA_ERR_INVALID_ARGUMENT
    assert lib.gqa_prefill_bf16(fake, fake, fake, fake, None, None, 1, 128, 32, 8, 128, 0, 8, -1.0, 1, None) == \
        E.GQA_ERR_INVALID_ARGUMENT
    # misaligned
    assert lib.gqa_prefill_bf16(mis, fake, fake, fake, None, None, 1, 128, 32, 8, 128, 0, 8, 0.1, 1, None) == \
        E.GQA_ERR_MISALIGNED
    # decode: workspace sizing and checks
    assert lib.gqa_decode_workspace_size(64, 32, 32768, 0) == 64 * 32 * 16 * 130 * 4
    assert lib.gqa_decode_workspace_size(0, 32, 1, 0) == 0
    assert lib.gqa_decode_bf16(fake, fake, fake, fake, None, None, None, fake, None, 0, 2, 64, 32, 8, 128, 0, 8, 0,
                               0.1, 0, None) == E.GQA_ERR_WORKSPACE
    assert lib.gqa_decode_bf16(fake, fake, fake, fake, None, None, None, fake, fake, 1 << 30, 2, 64, 32, 8, 128, 0, 8,
                               96, 0.1, 0, None) == E.GQA_ERR_INVALID_ARGUMENT  # split not a multiple of 64
    # stage kernels and the HLS-mask ABI
    assert lib.gqa_attention_mask_bf16(fake, fake, 0, 128, 1, 0xFF80, None) == E.GQA_ERR_INVALID_ARGUMENT
    assert lib.gqa_attention_mask_bf16(None, fake, 4, 128, 1, 0xFF80, None) == E.GQA_ERR_INVALID_ARGUMENT
    assert lib.gqa_rope_bf16(fake, fake, fake, fake, 1, 4, 127, 0, None) == E.GQA_ERR_INVALID_ARGUMENT
    assert lib.gqa_rope_cache_bf16(fake, fake, 8, 128, 0, -1.0, None) == E.GQA_ERR_INVALID_ARGUMENT
    assert lib.gqa_scores_bf16(fake, fake, fake, 1, 6, 4, 8, 128, 0.1, None) == E.GQA_ERR_INVALID_ARGUMENT
    assert lib.gqa_softmax_bf16(fake, fake, 0, 8, None) == E.GQA_ERR_INVALID_ARGUMENT
    assert lib.gqa_pv_bf16(fake, fake, None, 1, 4, 1, 8, 128, None) == E.GQA_ERR_INVALID_ARGUMENT
    # projections
    assert lib.gqa_gemm_bf16(None, fake, fake, 64, 64, 64, 64, 64, 64, 0, None) == E.GQA_ERR_INVALID_ARGUMENT
    assert lib.gqa_gemm_bf16(fake, fake, fake, 64, 64, 64, 32, 64, 64, 0, None) == E.GQA_ERR_INVALID_ARGUMENT  # lda < K
    assert lib.gqa_gemm_bf16(fake, fake, fake, 64, 64, 64, 64, 64, 64, 8, None) == E.GQA_ERR_INVALID_ARGUMENT  # flag
    assert lib.gqa_gemm_bf16(fake, fake, fake, 64, 64, 100, 100, 100, 64, 0, None) == E.GQA_ERR_MISALIGNED
    assert lib.gqa_gemm_bf16(mis, fake, fake, 64, 64, 64, 64, 64, 64, 0, None) == E.GQA_ERR_MISALIGNED
    assert lib.gqa_qkv_proj_bf16(fake, fake, fake, fake, fake, fake, fake, None, None, 1, 64, 4096, 32, 8, 128, 0,
                                 E.GQA_FLAG_ROPE_Q, None) == E.GQA_ERR_INVALID_ARGUMENT  # rope without tables
    assert lib.gqa_qkv_proj_bf16(fake, fake, fake, fake, fake, fake, fake, None, None, 1, 64, 4096, 32, 8, 64, 0,
                                 0, None) == E.GQA_ERR_UNSUPPORTED  # head_dim
    assert lib.gqa_qkv_proj_bf16(fake, fake, fake, fake, fake, fake, fake, None, None, 2, 100, 4096, 32, 8, 128, 0,
                                 0, None) == E.GQA_ERR_UNSUPPORTED  # batched S not a multiple of 128
    assert lib.gqa_o_proj_bf16(fake, fake, fake, 1, 64, 32, 128, 4096, 1024, 0, None) == \
        E.GQA_ERR_INVALID_ARGUMENT  # ldw narrower than the heads
    assert lib.gqa_cast_f32_bf16(None, fake, 16, None) == E.GQA_ERR_INVALID_ARGUMENT
    assert lib.gqa_cast_f32_bf16(fake, fake, 0, None) == E.GQA_OK


def test_python_wrappers_refuse_cpu_tensors():
    torch = pytest.importorskip("torch")
    from llama3_8b_attention_optimize_b200 import kernels
    q = torch.zeros(1, 4, 16, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        kernels.prefill(q, q[:, :1], q[:, :1])
