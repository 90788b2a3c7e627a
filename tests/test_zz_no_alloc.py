"""The allocation-free decode entry point (gqa_decode_bf16_noalloc).

It exists for callers that cannot allocate device memory -- a plugin host that
passes only its input/output buffers, a serving loop that must not call
cudaMalloc/cudaFree because they synchronise the device, or a process whose
memory pool is reserved in advance.  Its split-KV partials live in a fixed
16 MiB scratch array inside the library instead of a caller workspace.

This file runs last (collection order), so a failure here never hides another
test's result.  It calls the entry point through the C ABI several times in a
row (each call reuses the scratch left by the one before, with a different
shape) and requires each output to be bit-identical to the workspace entry
point gqa_decode_bf16: both run the same kernels with the same split, so any
difference -- even one far below the decode tolerance of max-abs 1e-2 /
mean-abs 1e-3 -- would be a scratch-aliasing bug.
"""
import ctypes

import numpy as np
import pytest
import torch

from llama3_8b_attention_optimize_b200 import _lib, kernels
from tests._util import randn_bf16

pytestmark = pytest.mark.gpu


def _noalloc(lib, q, kc, vc, lens, out, split_len=0, q_pos=None, cos=None, sin=None):
    B, Hq, d = q.shape
    Hkv, Lmax = kc.shape[1], kc.shape[2]
    flags = kernels.GQA_FLAG_ROPE_Q if q_pos is not None else 0
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    return lib.gqa_decode_bf16_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), ptr(q_pos),
                                       ptr(cos), ptr(sin), out.data_ptr(), B, Lmax, Hq, Hkv, d, 0, Hkv, split_len,
                                       kernels.default_scale(d), flags, torch.cuda.current_stream().cuda_stream)


def _case(B, Lmax, lens_np, seed, split_len=0, rope=False):
    Hq, Hkv = 32, 8
    q = randn_bf16((B, Hq, 128), seed)
    kc = randn_bf16((B, Hkv, Lmax, 128), seed + 1)
    vc = randn_bf16((B, Hkv, Lmax, 128), seed + 2)
    lens = torch.from_numpy(np.asarray(lens_np, np.int32)).cuda()
    extra = {}
    if rope:
        cos, sin = kernels.rope_cache(Lmax + 1)
        extra = dict(q_pos=lens.clone(), cos=cos, sin=sin)
    return q, kc, vc, lens, split_len, extra


def test_noalloc_decode_is_bit_identical_to_workspace_entry_point():
    lib = _lib.load()
    assert lib.gqa_decode_noalloc_scratch_bytes() == 16 << 20
    cases = [
        _case(4, 3000, [3000, 1, 1500, 2049], 7),
        _case(2, 1024, [700, 1024], 8),
        _case(3, 2500, [2500, 300, 1777], 9, split_len=256),          # explicit split length
        _case(2, 4096, [4000, 2], 10, rope=True),                      # q rotated at q_pos in the kernel
        _case(4, 3000, [3000, 1, 1500, 2049], 7),                      # first shape again, after the others
    ]
    stream = torch.cuda.current_stream().cuda_stream
    for q, kc, vc, lens, split_len, extra in cases:
        ref = kernels.decode(q, kc, vc, lens, split_len=split_len, **extra)
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(lib, q, kc, vc, lens, out, split_len=split_len, **extra)
        assert rc == 0, _lib.strerror(rc)
        site = ctypes.c_int(0)
        assert lib.gqa_device_check(stream, ctypes.byref(site)) == 0, hex(site.value)
        assert torch.isfinite(out.float()).all()
        assert torch.equal(out, ref)


def test_noalloc_rejects_requests_beyond_the_scratch():
    lib = _lib.load()
    B, Hq, Hkv, Lmax = 64, 32, 8, 32768  # needs 34 MiB of partials at the default split
    assert kernels.decode_workspace_bytes(B, Hq, Lmax) > lib.gqa_decode_noalloc_scratch_bytes()
    q = torch.zeros(B, Hq, 128, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(B, Hkv, 64, 128, dtype=torch.bfloat16, device="cuda")  # never read: rejected first
    lens = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.zeros_like(q)
    rc = lib.gqa_decode_bf16_noalloc(q.data_ptr(), kc.data_ptr(), kc.data_ptr(), lens.data_ptr(), None, None, None,
                                     out.data_ptr(), B, Lmax, Hq, Hkv, 128, 0, Hkv, 0, 0.088, 0,
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.GQA_ERR_WORKSPACE
