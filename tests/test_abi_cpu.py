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


def test_paged_cache_entry_points_validate_on_host(lib):
    E = _lib
    fake = ctypes.c_void_p(0x1000)
    # decode over pages: page_size / split not multiples of 128, null table, bad head_dim
    args = dict(max_pages=4, page_size=128, num_pages=8, B=2, Hq=32, Hkv=8, d=128, split=0, flags=0)

    def dec(**kw):
        a = {**args, **kw}
        return lib.gqa_decode_paged_bf16(fake, fake, fake, kw.get("table", fake), a["max_pages"], a["page_size"],
                                         a["num_pages"], fake, None, None, None, fake, fake, 1 << 30, a["B"], a["Hq"],
                                         a["Hkv"], a["d"], 0, a["Hkv"], a["split"], 0.088, a["flags"], None)

    assert dec(page_size=64) == E.GQA_ERR_UNSUPPORTED
    assert dec(split=192) == E.GQA_ERR_UNSUPPORTED
    assert dec(table=None) == E.GQA_ERR_INVALID_ARGUMENT
    assert dec(d=64) == E.GQA_ERR_UNSUPPORTED
    assert dec(num_pages=0) == E.GQA_ERR_INVALID_ARGUMENT
    assert dec(flags=2) == E.GQA_ERR_INVALID_ARGUMENT  # ROPE_Q without tables / q_pos
    assert dec(flags=4) == E.GQA_ERR_INVALID_ARGUMENT

    def app(**kw):
        a = dict(table=fake, max_pages=4, page_size=16, num_pages=8, B=2, Hkv=8, n=3, d=128, max_len=0, flags=0)
        a.update(kw)
        return lib.gqa_kv_append_bf16(fake, fake, fake, fake, a["table"], a["max_pages"], a["page_size"],
                                      a["num_pages"], fake, None, None, None, a["B"], a["Hkv"], a["n"], a["d"],
                                      a["max_len"], a["flags"], None)

    assert app(d=64) == E.GQA_ERR_UNSUPPORTED
    assert app(n=0) == E.GQA_ERR_INVALID_ARGUMENT
    assert app(flags=4) == E.GQA_ERR_INVALID_ARGUMENT  # ROPE_K without tables
    assert app(flags=2) == E.GQA_ERR_INVALID_ARGUMENT
    assert app(table=None, max_len=0) == E.GQA_ERR_INVALID_ARGUMENT
    assert app(page_size=0) == E.GQA_ERR_INVALID_ARGUMENT
    mis = ctypes.c_void_p(0x1002)
    assert lib.gqa_kv_append_bf16(mis, fake, fake, fake, None, 0, 0, 0, fake, None, None, None, 2, 8, 3, 128, 64, 0,
                                  None) == E.GQA_ERR_MISALIGNED
    assert lib.gqa_strerror(E.GQA_ERR_DEVICE_INPUT)


def test_row_chunks_cover_rows_on_tile_boundaries():
    from llama3_8b_attention_optimize_b200.layer import row_chunks
    for S, n in [(4096, 4), (4096, 3), (300, 8), (128, 5), (1, 2), (4097, 4)]:
        ch = row_chunks(S, n)
        assert ch[0][0] == 0 and sum(c for _, c in ch) == S and len(ch) <= n
        assert all(a + c == b for (a, c), (b, _) in zip(ch, ch[1:]))
        assert all(s0 % 128 == 0 and c > 0 for s0, c in ch)
    with pytest.raises(ValueError):
        row_chunks(0, 2)
