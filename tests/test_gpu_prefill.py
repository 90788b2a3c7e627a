"""GPU parity of the fused tcgen05 prefill kernel against the oracle.

Tolerance (stated by the task for bf16 attention outputs): max-abs <= 1e-2 and
mean-abs <= 1e-3 against the exact (float64-accumulated) attention of the same
bf16 inputs after the golden RoPE.  Where the reference value is >= 2 in
magnitude a bf16 output cannot be closer than half an ulp (2^-8 at 2..4,
2^-7 at 4..8), so the per-element bound is max(1e-2, 1 bf16 ulp of the value);
the C1/C2/edge configs (N(0,1) inputs) never reach that regime.
"""
import os

import numpy as np
import pytest
import torch

from llama3_8b_attention_optimize_b200 import kernels
from oracle import golden as g
from tests._util import bf16_ulp_of, bf16_words, randn_bf16, report_ulps as _report, ulp_histogram, words_to_bf16

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
THETA = 500000.0


def _rotated_words(x: torch.Tensor, S: int):
    cos, sin = g.rope_table(S, 128, THETA)
    w = bf16_words(x)
    return np.stack([g.rope_apply(w[b], cos, sin) for b in range(w.shape[0])])


def _check_rows(out: torch.Tensor, qr, kr, vw, rows_per_batch, causal=True, tag=""):
    """Compare sampled (batch, head, pos) rows of `out` with exact attention."""
    got = bf16_words(out)
    errs, ulps = [], []
    for b, (heads, pos) in enumerate(rows_per_batch):
        ref = g.attention_rows(qr[b], kr[b], vw[b], heads, pos, causal=causal)
        sel = got[b][heads, pos]
        gf = g.bf16_words_to_f32(sel)
        err = np.abs(gf - ref)
        allow = np.maximum(1e-2, bf16_ulp_of(ref))
        assert np.all(err <= allow), f"{tag}: max err {err.max()} at b={b}"
        errs.append(err)
        ulps.append(ulp_histogram(sel, g.to_bf16_words(ref)))
    e = np.concatenate([x.reshape(-1) for x in errs])
    assert e.mean() <= 1e-3, f"{tag}: mean abs err {e.mean()}"
    return float(e.max()), float(e.mean()), ulps


def _all_rows(Hq, S):
    heads = np.repeat(np.arange(Hq), S)
    pos = np.tile(np.arange(S), Hq)
    return heads, pos


def test_fpga_slice_golden_output():
    fs = dict(np.load(os.path.join(HERE, "golden", "fpga_slice.npz")))
    q = words_to_bf16(fs["q_before_rope"])[None]
    k = words_to_bf16(fs["k_before_rope"])[None]
    v = words_to_bf16(fs["v"])[None]
    cos, sin = kernels.rope_cache(128)
    out = kernels.prefill(q, k, v, cos, sin, causal=True, rope_q=True, rope_k=True)
    kernels.device_check()
    got = g.bf16_words_to_f32(bf16_words(out)[0])
    gold = g.bf16_words_to_f32(fs["attn_out_per_head"])
    assert np.abs(got - gold).max() <= 1e-2 and np.abs(got - gold).mean() <= 1e-3
    # against the exact result the kernel is at least as close as the golden's own
    # bf16-staged pipeline (which rounds scores and weights to bf16 on the way)
    heads, pos = _all_rows(4, 128)
    exact = g.attention_rows(fs["q_after_rope"], fs["k_after_rope"], fs["v"], heads, pos).reshape(4, 128, 128)
    assert np.abs(got - exact).mean() <= np.abs(gold - exact).mean()
    assert np.abs(got - exact).max() <= np.abs(gold - exact).max()
    # ulp counts are dominated by outputs near zero (tiny absolute error); the bound is
    # a regression guard, the tolerance proper is the absolute one above
    hist = ulp_histogram(bf16_words(out)[0], g.to_bf16_words(exact))
    assert hist["0"] + hist["1"] >= 0.85, hist


def test_c1_config_all_rows_vs_oracle():
    B, Hq, Hkv, S = 1, 32, 8, 128
    q = randn_bf16((B, Hq, S, 128), 2026)
    k = randn_bf16((B, Hkv, S, 128), 2027)
    v = randn_bf16((B, Hkv, S, 128), 2028)
    cos, sin = kernels.rope_cache(S)
    out = kernels.prefill(q, k, v, cos, sin, rope_q=True, rope_k=True)
    kernels.device_check()
    qr, kr, vw = _rotated_words(q, S), _rotated_words(k, S), bf16_words(v)
    mx, mean, ulps = _check_rows(out, qr, kr, vw, [_all_rows(Hq, S)], tag="C1")
    _report("prefill_c1_all_rows", ulps)
    # and against the bf16-staged golden pipeline (oracle restatement of run_full_attention)
    # The golden's bf16-staged pipeline rounds scores (|s| up to ~5 here) and weights to
    # bf16, which moves it up to ~1.6e-2 from the exact result; the kernel is held to
    # 1e-2 of the exact result above and must be closer to it than the golden is.
    st = g.stages(bf16_words(q)[0], bf16_words(k)[0], vw[0])
    gold = g.bf16_words_to_f32(st["attn_out_per_head"])
    got = g.bf16_words_to_f32(bf16_words(out)[0])
    exact = g.attention_rows(qr[0], kr[0], vw[0], *_all_rows(Hq, S)).reshape(Hq, S, 128)
    assert np.abs(got - gold).max() <= 2.5e-2 and np.abs(got - gold).mean() <= 1e-3
    assert np.abs(got - exact).mean() <= np.abs(gold - exact).mean()
    # ulp counts are dominated by outputs near zero (tiny absolute error); the bound is
    # a regression guard, the tolerance proper is the absolute one above
    hist = ulp_histogram(bf16_words(out)[0], g.to_bf16_words(exact))
    assert hist["0"] + hist["1"] >= 0.85, hist


EDGE_CASES = [
    # (B, S, causal, rope)
    (1, 1, True, True), (2, 7, True, False), (1, 31, True, True), (1, 32, True, True), (2, 33, True, True),
    (1, 63, False, True), (1, 64, True, True), (1, 65, True, False), (1, 127, True, True), (1, 129, False, True),
    (3, 200, True, True), (1, 255, True, True), (1, 257, False, False), (1, 384, True, True),
]


@pytest.mark.parametrize("B,S,causal,rope", EDGE_CASES)
def test_edge_shapes_vs_oracle(B, S, causal, rope):
    Hq, Hkv = 8, 2
    q = randn_bf16((B, Hq, S, 128), 11 + S)
    k = randn_bf16((B, Hkv, S, 128), 12 + S)
    v = randn_bf16((B, Hkv, S, 128), 13 + S)
    if rope:
        cos, sin = kernels.rope_cache(S)
        out = kernels.prefill(q, k, v, cos, sin, causal=causal, rope_q=True, rope_k=True)
        qr, kr = _rotated_words(q, S), _rotated_words(k, S)
    else:
        out = kernels.prefill(q, k, v, causal=causal)
        qr, kr = bf16_words(q), bf16_words(k)
    kernels.device_check()
    _check_rows(out, qr, kr, bf16_words(v), [_all_rows(Hq, S)] * B, causal=causal, tag=f"S={S}")


@pytest.mark.parametrize("B,Hkv,S,kv_heads", [(2, 8, 4800, None), (3, 2, 1100, None), (3, 2, 1100, (1, 1))])
def test_banded_unit_order_covers_every_block(B, Hkv, S, kv_heads):
    """Unit order: bands of 16 query blocks per (sequence, kv head) when the pairs are many
    and the problem has enough rounds, else plain heaviest-first order.

    Batch 2 x 8 kv heads at S = 4800 (75 query blocks: 4 full bands and a partial one,
    16 pairs, 1200 units) takes the banded order; batch 3 x 2 kv heads at S = 1100, with
    all or a subset of the kv heads, takes the plain one.  Every output row must be
    written once and match exact attention: the output starts as NaN, and one row of
    every query block of every (sequence, head) is checked against the oracle.
    """
    Hq = 4 * Hkv
    q = randn_bf16((B, Hq, S, 128), 41)
    k = randn_bf16((B, Hkv, S, 128), 42)
    v = randn_bf16((B, Hkv, S, 128), 43)
    cos, sin = kernels.rope_cache(S)
    out = torch.full((B, Hq, S, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
    kernels.prefill(q, k, v, cos, sin, rope_q=True, rope_k=True, kv_heads=kv_heads, out=out)
    kernels.device_check()
    h0, hn = (0, Hq) if kv_heads is None else (kv_heads[0] * 4, kv_heads[1] * 4)
    assert torch.isfinite(out[:, h0:h0 + hn].float()).all()
    if kv_heads is not None:
        assert torch.isnan(out[:, :h0].float()).all() and torch.isnan(out[:, h0 + hn:].float()).all()
    qr, kr = _rotated_words(q, S), _rotated_words(k, S)
    rows = []
    for b in range(B):
        heads, pos = [], []
        for h in range(h0, h0 + hn):
            for qb in range((S + 63) // 64):
                p = qb * 64 + (7 * h + 13 * b + 5 * qb) % 64
                if p < S:
                    heads.append(h)
                    pos.append(p)
        rows.append((np.array(heads), np.array(pos)))
    _check_rows(out, qr, kr, bf16_words(v), rows, tag=f"banded kv_heads={kv_heads}")


def test_fused_rope_equals_prerotated_inputs():
    B, Hq, Hkv, S = 2, 32, 8, 320
    q = randn_bf16((B, Hq, S, 128), 1)
    k = randn_bf16((B, Hkv, S, 128), 2)
    v = randn_bf16((B, Hkv, S, 128), 3)
    cos, sin = kernels.rope_cache(S)
    fused = kernels.prefill(q, k, v, cos, sin, rope_q=True, rope_k=True)
    pre = kernels.prefill(kernels.rope(q, cos, sin), kernels.rope(k, cos, sin), v)
    kernels.device_check()
    assert torch.equal(fused, pre)


def test_c2_config_sampled_rows():
    B, Hq, Hkv, S = 1, 32, 8, 2048
    q = randn_bf16((B, Hq, S, 128), 7)
    k = randn_bf16((B, Hkv, S, 128), 8)
    v = randn_bf16((B, Hkv, S, 128), 9)
    cos, sin = kernels.rope_cache(S)
    out = kernels.prefill(q, k, v, cos, sin, rope_q=True, rope_k=True)
    kernels.device_check()
    rng = np.random.default_rng(0)
    heads = np.concatenate([np.arange(Hq), np.arange(Hq), rng.integers(0, Hq, 448)])
    pos = np.concatenate([np.zeros(Hq, int), np.full(Hq, S - 1), rng.integers(0, S, 448)])
    _check_rows(out, _rotated_words(q, S), _rotated_words(k, S), bf16_words(v), [(heads, pos)], tag="C2")


@pytest.mark.slow
def test_c3_config_sampled_rows_and_properties():
    B, Hq, Hkv, S = 4, 32, 8, 8192
    q = randn_bf16((B, Hq, S, 128), 100, 2.5)
    k = randn_bf16((B, Hkv, S, 128), 101, 2.5)
    v = randn_bf16((B, Hkv, S, 128), 102)
    cos, sin = kernels.rope_cache(S)
    out = kernels.prefill(q, k, v, cos, sin, rope_q=True, rope_k=True)
    kernels.device_check()
    assert torch.isfinite(out.float()).all()
    rng = np.random.default_rng(1)
    rows = []
    for b in range(B):
        heads = rng.integers(0, Hq, 96)
        pos = np.concatenate([[0, 1, 127, 128, S - 1], rng.integers(0, S, 91)])
        rows.append((heads, pos))
    qr, kr, vw = _rotated_words(q, S), _rotated_words(k, S), bf16_words(v)
    _, _, ulps = _check_rows(out, qr, kr, vw, rows, tag="C3")
    _report("prefill_c3_fused_sampled_rows", ulps)

    # the benchmark's timed mode: K rotated by its own launch, Q inside the fused kernel
    # (PrefillSession.run_device, rope="prepass_k"), checked against the oracle itself
    from llama3_8b_attention_optimize_b200.session import PrefillSession
    sess = PrefillSession(B, S, Hq, Hkv, rope="prepass_k")
    sess.q.copy_(q)
    sess.k.copy_(k)
    sess.v.copy_(v)
    bench_out = sess.run_device().clone()
    kernels.device_check()
    _, _, ulps = _check_rows(bench_out, qr, kr, vw, rows, tag="C3 prepass_k")
    _report("prefill_c3_bench_mode_sampled_rows", ulps)
    assert torch.equal(bench_out, out)
    del sess, bench_out

    # KV-head shards computed separately are bit-identical to the full run
    sharded = torch.full_like(out, float("nan"))
    for kvh in range(Hkv):
        kernels.prefill(q, k, v, cos, sin, rope_q=True, rope_k=True, kv_heads=(kvh, 1), out=sharded)
    assert torch.equal(sharded, out)

    # batch independence
    one = kernels.prefill(q[2:3].contiguous(), k[2:3].contiguous(), v[2:3].contiguous(), cos, sin,
                          rope_q=True, rope_k=True)
    assert torch.equal(one[0], out[2])

    # causality: perturbing keys/values at positions >= 6000 leaves earlier rows bit-identical
    k2, v2 = k.clone(), v.clone()
    k2[:, :, 6000:] = -k2[:, :, 6000:]
    v2[:, :, 6000:] = 3.0
    out2 = kernels.prefill(q, k2, v2, cos, sin, rope_q=True, rope_k=True)
    kernels.device_check()
    assert torch.equal(out2[:, :, :6000], out[:, :, :6000])
    assert not torch.equal(out2[:, :, 6000:], out[:, :, 6000:])


def test_kv_head_shard_writes_only_its_heads():
    B, Hq, Hkv, S = 2, 32, 8, 256
    q = randn_bf16((B, Hq, S, 128), 21)
    k = randn_bf16((B, Hkv, S, 128), 22)
    v = randn_bf16((B, Hkv, S, 128), 23)
    out = torch.full((B, Hq, S, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
    kernels.prefill(q, k, v, kv_heads=(2, 3), out=out)
    kernels.device_check()
    inside = out[:, 8:20].float()
    assert torch.isfinite(inside).all()
    assert torch.isnan(out[:, :8].float()).all() and torch.isnan(out[:, 20:].float()).all()
    full = kernels.prefill(q, k, v)
    assert torch.equal(full[:, 8:20], out[:, 8:20])


def test_prefill_stream_overlapped_host_steps_match_device_results():
    """PrefillStream: each step's host output equals the device-resident result of its inputs."""
    from llama3_8b_attention_optimize_b200.session import PrefillStream
    B, Hq, Hkv, S = 1, 32, 8, 256
    pipe = PrefillStream(B, S, Hq, Hkv)
    steps, refs = [], []
    cos, sin = kernels.rope_cache(S)
    for i in range(5):
        q = randn_bf16((B, Hq, S, 128), 300 + i)
        k = randn_bf16((B, Hkv, S, 128), 400 + i)
        v = randn_bf16((B, Hkv, S, 128), 500 + i)
        refs.append(kernels.prefill(q, kernels.rope(k, cos, sin), v, cos, sin, rope_q=True).cpu())
        steps.append((q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory(),
                      torch.empty(B, Hq, S, 128, dtype=torch.bfloat16).pin_memory()))
    pipe.run(steps)
    torch.cuda.synchronize()
    kernels.device_check()
    for (_, _, _, out), ref in zip(steps, refs):
        assert torch.equal(out, ref)


def test_prefill_session_graph_replay_equals_direct_launches():
    """PrefillSession.capture(): replaying the recorded step (K pre-pass + fused kernel)
    gives the direct launches' output bit for bit, also after new inputs are copied into
    the session's buffers in place."""
    from llama3_8b_attention_optimize_b200.session import PrefillSession
    sess = PrefillSession(1, 2048, 32, 8)
    sess.q.copy_(randn_bf16(sess.shape_q, 61))
    sess.k.copy_(randn_bf16(sess.shape_kv, 62))
    sess.v.copy_(randn_bf16(sess.shape_kv, 63))
    graph = sess.capture()
    for seed in (0, 10):
        sess.q.copy_(randn_bf16(sess.shape_q, 71 + seed))
        sess.k.copy_(randn_bf16(sess.shape_kv, 72 + seed))
        sess.v.copy_(randn_bf16(sess.shape_kv, 73 + seed))
        direct = sess.run_device().clone()
        sess.o.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        kernels.device_check()
        assert torch.equal(sess.o, direct)
    del graph
