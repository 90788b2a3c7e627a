"""GPU parity of the split-KV decode kernel against exact attention from the oracle.

Tolerance: max-abs <= max(1e-2, 1 bf16 ulp of the reference) and mean-abs <= 1e-3
against float64-accumulated attention over keys [0, lens[b]).
"""
import numpy as np
import pytest
import torch

from llama3_8b_attention_optimize_b200 import kernels
from oracle import golden as g
from tests._util import bf16_ulp_of, bf16_words, randn_bf16, report_ulps, ulp_histogram

pytestmark = pytest.mark.gpu


def _reference(q, kc, vc, lens, batches, heads):
    """Exact decode outputs for selected (b, h): q [B,Hq,d] (already rotated)."""
    qw, out = bf16_words(q), []
    for b, h in zip(batches, heads):
        L = int(lens[b])
        kw = bf16_words(kc[b, h // 4 : h // 4 + 1, :L])
        vw = bf16_words(vc[b, h // 4 : h // 4 + 1, :L])
        out.append(g.attention_rows(qw[b, h][None, None], kw, vw, [0], [0], causal=False)[0])
    return np.stack(out)


def _check(out, ref, batches, heads):
    sel = bf16_words(out)[batches, heads]
    got = g.bf16_words_to_f32(sel)
    err = np.abs(got - ref)
    assert np.all(err <= np.maximum(1e-2, bf16_ulp_of(ref))), err.max()
    assert err.mean() <= 1e-3, err.mean()
    return ulp_histogram(sel, g.to_bf16_words(ref))


@pytest.mark.parametrize("B,Lmax,split", [(3, 100, 0), (2, 1000, 64), (4, 3000, 256), (2, 130, 128)])
def test_decode_small_all_heads(B, Lmax, split):
    Hq, Hkv = 32, 8
    q = randn_bf16((B, Hq, 128), 1 + B)
    kc = randn_bf16((B, Hkv, Lmax, 128), 2 + B)
    vc = randn_bf16((B, Hkv, Lmax, 128), 3 + B)
    rng = np.random.default_rng(Lmax)
    lens_np = rng.integers(1, Lmax + 1, B).astype(np.int32)
    lens_np[0] = Lmax
    lens = torch.from_numpy(lens_np).cuda()
    out = kernels.decode(q, kc, vc, lens, split_len=split)
    kernels.device_check()
    bs = np.repeat(np.arange(B), Hq)
    hs = np.tile(np.arange(Hq), B)
    _check(out, _reference(q, kc, vc, lens_np, bs, hs), bs, hs)


def test_decode_rope_q_in_kernel_matches_prerotated():
    B, Hq, Hkv, Lmax = 4, 32, 8, 700
    q = randn_bf16((B, Hq, 128), 41)
    kc = randn_bf16((B, Hkv, Lmax, 128), 42)
    vc = randn_bf16((B, Hkv, Lmax, 128), 43)
    lens = torch.tensor([700, 1, 333, 64], dtype=torch.int32, device="cuda")
    cos, sin = kernels.rope_cache(1024)
    fused = kernels.decode(q, kc, vc, lens, q_pos=lens, cos=cos, sin=sin)
    qr = torch.empty_like(q)
    for b in range(B):  # rotate row b at position lens[b]
        qr[b] = kernels.rope(q[b : b + 1].unsqueeze(2).contiguous(), cos, sin, pos0=int(lens[b]))[0, :, 0]
    pre = kernels.decode(qr, kc, vc, lens)
    kernels.device_check()
    assert torch.equal(fused, pre)


def test_decode_kv_shard_and_canary():
    B, Hq, Hkv, Lmax = 2, 32, 8, 512
    q = randn_bf16((B, Hq, 128), 51)
    kc = randn_bf16((B, Hkv, Lmax, 128), 52)
    vc = randn_bf16((B, Hkv, Lmax, 128), 53)
    lens = torch.tensor([512, 300], dtype=torch.int32, device="cuda")
    out = torch.full((B, Hq, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
    kernels.decode(q, kc, vc, lens, kv_heads=(4, 2), out=out)
    kernels.device_check()
    assert torch.isfinite(out[:, 16:24].float()).all()
    assert torch.isnan(out[:, :16].float()).all() and torch.isnan(out[:, 24:].float()).all()
    full = kernels.decode(q, kc, vc, lens)
    assert torch.equal(full[:, 16:24], out[:, 16:24])


@pytest.mark.slow
def test_decode_c5_config_sampled():
    B, Hq, Hkv, Lmax = 64, 32, 8, 32768
    gen = torch.Generator().manual_seed(5)
    lens_np = torch.randint(1024, 32769, (B,), generator=gen).numpy().astype(np.int32)
    q = randn_bf16((B, Hq, 128), 61)
    kc = randn_bf16((B, Hkv, Lmax, 128), 62)
    vc = randn_bf16((B, Hkv, Lmax, 128), 63)
    lens = torch.from_numpy(lens_np).cuda()
    out = kernels.decode(q, kc, vc, lens)
    kernels.device_check()
    rng = np.random.default_rng(2)
    bs = rng.integers(0, B, 48)
    hs = rng.integers(0, Hq, 48)
    report_ulps("decode_c5_sampled_rows", _check(out, _reference(q, kc, vc, lens_np, bs, hs), bs, hs))
    # split length does not change the result beyond rounding
    out2 = kernels.decode(q, kc, vc, lens, split_len=4096)
    d = (out.float() - out2.float()).abs()
    assert d.max().item() <= 2e-2 and d.mean().item() <= 1e-4


@pytest.mark.parametrize("split", [0, 64, 384])
def test_decode_ignores_non_finite_cache_past_lens(split):
    """Cache rows at or past lens[b] may hold anything (NaN, inf): they must not reach the output."""
    B, Hq, Hkv, Lmax = 4, 32, 8, 1000
    q = randn_bf16((B, Hq, 128), 71)
    kc = randn_bf16((B, Hkv, Lmax, 128), 72)
    vc = randn_bf16((B, Hkv, Lmax, 128), 73)
    lens_np = np.array([1000, 1, 129, 0], dtype=np.int32)
    lens = torch.from_numpy(lens_np).cuda()
    clean = kernels.decode(q, kc, vc, lens, split_len=split)
    kp, vp = kc.clone(), vc.clone()
    for b, L in enumerate(lens_np):
        kp[b, :, L:] = float("nan")
        vp[b, :, L:] = float("inf") if b % 2 else float("nan")
    dirty = kernels.decode(q, kp, vp, lens, split_len=split)
    kernels.device_check()
    assert torch.equal(clean, dirty)
    assert torch.isfinite(dirty.float()).all()
    assert (dirty[3].float() == 0).all()  # an empty sequence gives zeros
    bs = np.repeat(np.arange(3), Hq)
    hs = np.tile(np.arange(Hq), 3)
    _check(dirty, _reference(q, kc, vc, lens_np, bs, hs), bs, hs)
