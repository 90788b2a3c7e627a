"""The allocation-free decode entry point (gqa_decode_bf16_noalloc).

It exists for callers that cannot allocate device memory -- a plugin host that
passes only its input/output buffers, a serving loop that must not call
cudaMalloc/cudaFree because they synchronise the device, or a process whose
memory pool is reserved in advance.  Its split-KV partials live in a fixed
16 MiB scratch array inside the library instead of a caller workspace.

This file runs last (collection order), so a failure here never hides another
test's result.  It calls the entry point through the C ABI twice in a row (the
second call reuses the scratch left by the first) and compares each output with
the workspace entry point gqa_decode_bf16 under the decode tests' tolerance.
"""
import ctypes

import numpy as np
import pytest
import torch

from llama3_8b_attention_optimize_b200 import _lib, kernels
from tests._util import randn_bf16

pytestmark = pytest.mark.gpu


def _noalloc(lib, q, kc, vc, lens, out, split_len=0):
    B, Hq, d = q.shape
    Hkv, Lmax = kc.shape[1], kc.shape[2]
    return lib.gqa_decode_bf16_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), None, None, None,
                                       out.data_ptr(), B, Lmax, Hq, Hkv, d, 0, Hkv, split_len,
                                       kernels.default_scale(d), 0, torch.cuda.current_stream().cuda_stream)


def _close(a: torch.Tensor, b: torch.Tensor):
    # decode tolerance: max-abs <= 1e-2, mean-abs <= 1e-3 (here the two paths share kernels)
    d = (a.float() - b.float()).abs()
    assert d.max().item() <= 1e-2 and d.mean().item() <= 1e-3


def test_noalloc_decode_matches_workspace_entry_point_twice():
    lib = _lib.load()
    assert lib.gqa_decode_noalloc_scratch_bytes() == 16 << 20
    Hq, Hkv = 32, 8
    cases = [(4, 3000, np.array([3000, 1, 1500, 2049], np.int32), 7),
             (2, 1024, np.array([700, 1024], np.int32), 8)]
    for B, Lmax, lens_np, seed in cases:  # two calls in a row, different shapes
        q = randn_bf16((B, Hq, 128), seed)
        kc = randn_bf16((B, Hkv, Lmax, 128), seed + 1)
        vc = randn_bf16((B, Hkv, Lmax, 128), seed + 2)
        lens = torch.from_numpy(lens_np).cuda()
        ref = kernels.decode(q, kc, vc, lens)
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(lib, q, kc, vc, lens, out)
        assert rc == 0, _lib.strerror(rc)
        site = ctypes.c_int(0)
        assert lib.gqa_device_check(torch.cuda.current_stream().cuda_stream, ctypes.byref(site)) == 0
        assert torch.isfinite(out.float()).all()
        _close(out, ref)


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
