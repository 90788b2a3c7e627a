"""GPU parity of the projection GEMM (q/k/v and o_proj of the full layer).

Reference arithmetic: y = to_bf16(x @ W^T) with fp32 accumulation
(llama3_attention_golden_model.py:149-151, :193-194).  Accumulation order differs
from any CPU BLAS, so the check is against the float64 product: every bf16 output
lies within one bf16 ulp of it plus the fp32 accumulation allowance
2^-20 * sum_k |x_k w_k| (which only matters where the sum cancels to a tiny value --
plain sequential fp32 accumulation needs it too), and almost all outputs are the
correctly rounded value itself.
"""
import importlib.util
import os

import numpy as np
import pytest
import torch

from llama3_8b_attention_optimize_b200 import golden_model, kernels
from oracle import golden as g
from tests._util import bf16_ulp_of, bf16_words, randn_bf16, report_ulps, ulp_histogram, words_to_bf16

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


class Exact(np.ndarray):
    """float64 product carrying sum_k |x_k w_k| (the accumulation-error scale) as .absdot."""


def _exact(x: torch.Tensor, w: torch.Tensor, rows=None) -> np.ndarray:
    xa = x.float().cpu().double().numpy().reshape(-1, x.shape[-1])
    if rows is not None:
        xa = xa[rows]
    wa = w.float().cpu().double().numpy()
    out = (xa @ wa.T).view(Exact)
    out.absdot = np.abs(xa) @ np.abs(wa).T
    return out


def _reshape(e: np.ndarray, *shape, axes=None) -> np.ndarray:
    out = e.reshape(*shape) if axes is None else e.reshape(*shape).transpose(*axes)
    ad = e.absdot.reshape(*shape) if axes is None else e.absdot.reshape(*shape).transpose(*axes)
    out = np.ascontiguousarray(out).view(Exact)
    out.absdot = np.ascontiguousarray(ad)
    return out


def _check_bf16(got: torch.Tensor, exact: np.ndarray, min_exact: float = 0.97) -> dict:
    gw = bf16_words(got).reshape(exact.shape)
    ex = np.asarray(exact, dtype=np.float64)
    ew = g.to_bf16_words(ex.astype(np.float32))
    gf = g.bf16_words_to_f32(gw).astype(np.float64)
    err = np.abs(gf - ex)
    allow = bf16_ulp_of(ex) * 1.0001 + 2.0 ** -20 * exact.absdot
    assert np.all(err <= allow), (err - allow).max()
    assert np.mean(gw == ew) >= min_exact, np.mean(gw == ew)
    return ulp_histogram(gw, ew)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 200, 72), (257, 384, 520), (1024, 1024, 4096)])
def test_linear_vs_float64(M, N, K):
    x = randn_bf16((M, K), 11 + M)
    w = randn_bf16((N, K), 12 + N, scale=0.02)
    got = kernels.linear(x, w)
    kernels.device_check()
    _check_bf16(got, _exact(x, w))


@pytest.mark.parametrize("M,N,K", [(200, 96, 136), (512, 1024, 1024)])
def test_linear_fp32_output(M, N, K):
    x = randn_bf16((M, K), 21)
    w = randn_bf16((N, K), 22, scale=0.02)
    got = kernels.linear(x, w, out_f32=True)
    kernels.device_check()
    ex = _exact(x, w)
    assert np.all(np.abs(got.cpu().double().numpy() - ex) <= 2.0 ** -20 * ex.absdot + 1e-30)
    # the bf16 path is the rounding of the same sums
    assert torch.equal(kernels.cast_bf16(got), kernels.linear(x, w))


def test_linear_rejects_bad_arguments():
    x = randn_bf16((64, 100), 1)  # K = 100: rows not 16-byte aligned
    w = randn_bf16((64, 100), 2)
    with pytest.raises(kernels.GqaError):
        kernels.linear(x, w)


@pytest.mark.parametrize("B,S", [(1, 200), (2, 256)])
def test_qkv_proj_head_major_and_fused_rope(B, S):
    hidden, Hq, Hkv = 1024, 8, 2
    h = randn_bf16((B, S, hidden), 31)
    wq = randn_bf16((Hq * 128, hidden), 32, scale=0.02)
    wk = randn_bf16((Hkv * 128, hidden), 33, scale=0.02)
    wv = randn_bf16((Hkv * 128, hidden), 34, scale=0.02)
    q, k, v = kernels.qkv_proj(h, wq, wk, wv)
    kernels.device_check()
    for t, w, H in ((q, wq, Hq), (k, wk, Hkv), (v, wv, Hkv)):
        _check_bf16(t, _reshape(_exact(h, w), B, S, H, 128, axes=(0, 2, 1, 3)))
    cos, sin = kernels.rope_cache(S + 5)
    qr, kr, vr = kernels.qkv_proj(h, wq, wk, wv, cos, sin, rope_q=True, rope_k=True)
    kernels.device_check()
    # the rotation in the epilogue is the rope stage applied to the rounded projection
    assert torch.equal(qr, kernels.rope(q, cos, sin))
    assert torch.equal(kr, kernels.rope(k, cos, sin))
    assert torch.equal(vr, v)
    # position offset (a chunk of a longer sequence)
    qo, ko, _ = kernels.qkv_proj(h, wq, wk, wv, cos, sin, rope_q=True, rope_k=True, pos0=5)
    assert torch.equal(qo, kernels.rope(q, cos, sin, pos0=5))
    assert torch.equal(ko, kernels.rope(k, cos, sin, pos0=5))


def test_o_proj_reads_head_major_and_shards_sum():
    S, H, N = 384, 8, 512
    attn = randn_bf16((H, S, 128), 41, scale=0.5)
    wo = randn_bf16((N, H * 128), 42, scale=0.02)
    flat = attn.transpose(0, 1).contiguous().view(S, H * 128)  # reference :193
    ex = _exact(flat, wo)
    got = kernels.o_proj(attn, wo)
    kernels.device_check()
    _check_bf16(got, ex)
    # row-parallel shards (2 x 4 heads): fp32 partials summed, then one rounding
    parts = [kernels.o_proj(attn[h0:h0 + 4].contiguous(), wo, head_begin=h0, out_f32=True) for h0 in (0, 4)]
    total = kernels.cast_bf16(parts[0] + parts[1])
    kernels.device_check()
    _check_bf16(total, ex)


def _layer_inputs():
    spec = importlib.util.spec_from_file_location("make_fixtures", os.path.join(HERE, "golden", "make_fixtures.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.layer_inputs()


def test_full_layer_matches_reference_dump():
    """run_full_attention on the reference's own dump (seq 32, seeded weights)."""
    fx = np.load(os.path.join(HERE, "golden", "layer_s32.npz"))
    h, wq, wk, wv, wo = (words_to_bf16(w) for w in _layer_inputs())
    assert np.array_equal(bf16_words(h), fx["hidden_states_input"])
    for debug in (True, False):
        dump = golden_model.run_full_attention(h.float(), wq.float(), wk.float(), wv.float(), wo.float(),
                                               debug=debug)
        for key in ("q_before_rope", "k_before_rope", "v"):
            # two fp32 accumulation orders (ours, the reference's CPU matmul) of the same sums
            got = g.to_bf16_words(dump[key].cpu().numpy())
            gf, rf = g.bf16_words_to_f32(got), g.bf16_words_to_f32(fx[key])
            assert np.all(np.abs(gf - rf) <= bf16_ulp_of(rf) + 1e-4), key
            assert np.mean(got == fx[key]) >= 0.97, key
        ow = g.to_bf16_words(dump["final_output"].cpu().numpy())
        out, ref = g.bf16_words_to_f32(ow), g.bf16_words_to_f32(fx["final_output"])
        err = np.abs(out - ref)
        hist = ulp_histogram(ow, fx["final_output"])
        if debug:
            # staged path: the 1-ulp projection differences above flip some bf16 stage
            # roundings downstream (scores, softmax, PV): max(1e-2, 2 bf16 ulp) per element
            assert np.all(err <= np.maximum(1e-2, 2 * bf16_ulp_of(ref))), (err.max(), hist)
            assert err.mean() <= 1e-3, (err.mean(), hist)
            assert hist["0"] >= 0.6, hist
        else:
            # fused core: no bf16 rounding of scores / weights, so it sits closer to exact
            # attention than the staged golden; each half is held to its own bound
            attn = dump["attn_out_per_head"]
            qw, kw, vw = (g.to_bf16_words(dump[n].cpu().numpy()) for n in ("q_after_rope", "k_after_rope", "v"))
            Hq, S = qw.shape[0], qw.shape[1]
            rows = (np.repeat(np.arange(Hq), S), np.tile(np.arange(S), Hq))
            exact_attn = g.attention_rows(qw, kw, vw, *rows).reshape(Hq, S, 128)
            aerr = np.abs(attn.cpu().numpy() - exact_attn)
            assert np.all(aerr <= np.maximum(1e-2, bf16_ulp_of(exact_attn))) and aerr.mean() <= 1e-3
            flat = attn.to(torch.bfloat16).transpose(0, 1).contiguous().view(S, -1)
            fe = _exact(flat, wo)
            report_ulps("layer_s32_final_output_vs_float64_o_proj",
                        _check_bf16(dump["final_output"].to(torch.bfloat16), fe))
            # against the reference's staged result: both approximate the exact layer, and
            # the fused path is the closer of the two
            Hq, S = fx["q_after_rope"].shape[:2]
            rows = (np.repeat(np.arange(Hq), S), np.tile(np.arange(S), Hq))
            ea = g.attention_rows(fx["q_after_rope"], fx["k_after_rope"], fx["v"], *rows).reshape(Hq, S, 128)
            exact_final = ea.astype(np.float64).transpose(1, 0, 2).reshape(S, -1) @ \
                wo.float().cpu().double().numpy().T
            e_ours, e_gold = np.abs(out - exact_final).mean(), np.abs(ref - exact_final).mean()
            assert e_ours <= e_gold, (e_ours, e_gold)
            assert err.max() <= 6.25e-2 and err.mean() <= 5e-3, (err.mean(), err.max(), hist)
    # o_proj alone on the reference's own attention output: the GEMM bound
    attn_ref = words_to_bf16(fx["attn_out_per_head"])
    ow = g.to_bf16_words(kernels.o_proj(attn_ref, wo).float().cpu().numpy())
    out, ref = g.bf16_words_to_f32(ow), g.bf16_words_to_f32(fx["final_output"])
    assert np.all(np.abs(out - ref) <= bf16_ulp_of(ref) + 1e-4)
    assert np.mean(ow == fx["final_output"]) >= 0.97


@pytest.mark.slow
def test_c4_projection_shapes_sampled_rows():
    """Full-layer sizes (S=4096, hidden 4096): fused q/k/v and o_proj on sampled rows."""
    S, hidden = 4096, 4096
    h = randn_bf16((S, hidden), 51)
    wq = randn_bf16((4096, hidden), 52, scale=0.02)
    wk = randn_bf16((1024, hidden), 53, scale=0.02)
    wv = randn_bf16((1024, hidden), 54, scale=0.02)
    wo = randn_bf16((4096, 4096), 55, scale=0.02)
    q, k, v = kernels.qkv_proj(h, wq, wk, wv)
    attn = randn_bf16((32, S, 128), 56, scale=0.5)
    o = kernels.o_proj(attn, wo)
    kernels.device_check()
    rows = np.random.default_rng(0).choice(S, 48, replace=False)
    for t, w, H in ((q, wq, 32), (k, wk, 8), (v, wv, 8)):
        _check_bf16(t[:, rows].transpose(0, 1), _reshape(_exact(h, w, rows), len(rows), H, 128))
    flat = attn.transpose(0, 1).contiguous().view(S, 4096)
    report_ulps("c4_o_proj_sampled_rows_vs_float64", _check_bf16(o[rows], _exact(flat, wo, rows)))


def test_layer_session_matches_facade_and_shards_sum():
    """FullLayerSession (RoPE in the projection epilogue) == run_full_attention(debug=False)
    bit for bit; two row-parallel shards summed in fp32 agree to the GEMM bound."""
    from llama3_8b_attention_optimize_b200.layer import FullLayerSession
    S = 256
    h = randn_bf16((1, S, 4096), 61)
    ws = [randn_bf16(shp, 62 + i, scale=0.02) for i, shp in enumerate(((4096, 4096), (1024, 4096), (1024, 4096),
                                                                       (4096, 4096)))]
    sess = FullLayerSession(S)
    sess.set_weights(*ws)
    sess.h.copy_(h)
    out = sess.run_device().clone()
    dump = golden_model.run_full_attention(h[0], *ws, debug=False)
    kernels.device_check()
    assert torch.equal(out[0], dump["final_output"].to(torch.bfloat16))
    parts = []
    for r in range(2):
        sh = FullLayerSession(S, rank=r, world=2)
        sh.set_weights(*ws)
        sh.h.copy_(h)
        parts.append(sh.run_partial().clone())
    total = kernels.cast_bf16(parts[0] + parts[1])
    kernels.device_check()
    attn = sess.attn[0].transpose(0, 1).contiguous().view(S, -1)
    _check_bf16(total[0], _exact(attn, ws[3]))


def test_o_proj_rows_chunks_equal_full_call():
    """Row chunks of o_proj (the overlap pipeline's GEMM) are bit-identical to the full call,
    with and without a grid cap, in fp32 and bf16."""
    g0 = torch.Generator(device="cuda").manual_seed(77)
    Hq, S, N = 8, 700, 4096
    attn = (torch.randn(Hq, S, 128, generator=g0, device="cuda")).to(torch.bfloat16)
    wo = (torch.randn(N, 4096, generator=g0, device="cuda") * 0.02).to(torch.bfloat16)
    for f32 in (True, False):
        full = kernels.o_proj(attn, wo, head_begin=2, out_f32=f32)
        dt = torch.float32 if f32 else torch.bfloat16
        got = torch.full((S, N), float("nan"), dtype=dt, device="cuda")
        for (s0, n), cap in zip([(0, 128), (128, 384), (512, 188)], (0, 100, 7)):
            kernels.o_proj_rows(attn, wo, got, s0, n, head_begin=2, out_f32=f32, max_ctas=cap)
        kernels.device_check()
        assert torch.equal(got, full)
    # a chunk leaves the other rows untouched
    part = torch.full((S, N), 5.0, dtype=torch.float32, device="cuda")
    kernels.o_proj_rows(attn, wo, part, 256, 128, out_f32=True)
    kernels.device_check()
    assert torch.all(part[:256] == 5.0) and torch.all(part[384:] == 5.0)
    assert torch.equal(part[256:384], kernels.o_proj(attn, wo, out_f32=True)[256:384])


def test_cta_pair_tiles_equal_single_cta_tiles():
    """Row counts that divide into 256-row tiles run on CTA pairs (tcgen05.mma.cta_group::2,
    half of W per CTA); other row counts run on single CTAs.  Both accumulate the same
    products in the same order, so every row of a pair-tiled call equals the same row of
    single-CTA calls bit for bit (bf16 and fp32 outputs, with and without a grid cap)."""
    g0 = torch.Generator(device="cuda").manual_seed(78)
    Hq, S, N = 8, 1024, 4096
    attn = (torch.randn(Hq, S, 128, generator=g0, device="cuda")).to(torch.bfloat16)
    wo = (torch.randn(N, 4096, generator=g0, device="cuda") * 0.02).to(torch.bfloat16)
    for f32 in (True, False):
        full = kernels.o_proj(attn, wo, head_begin=1, out_f32=f32)  # 1024 rows: CTA pairs
        dt = torch.float32 if f32 else torch.bfloat16
        got = torch.full((S, N), float("nan"), dtype=dt, device="cuda")
        # chunks of 128 and 384 rows run on single CTAs, the 256-row chunk on a pair
        for (s0, n), cap in zip([(0, 128), (128, 384), (512, 256), (768, 128), (896, 128)], (0, 0, 10, 0, 5)):
            kernels.o_proj_rows(attn, wo, got, s0, n, head_begin=1, out_f32=f32, max_ctas=cap)
        kernels.device_check()
        assert torch.equal(got, full)
    x = (torch.randn(768, 4096, generator=g0, device="cuda")).to(torch.bfloat16)
    w = (torch.randn(512, 4096, generator=g0, device="cuda") * 0.02).to(torch.bfloat16)
    pair = kernels.linear(x, w)                                   # 768 rows: pairs
    single = torch.cat([kernels.linear(x[i:i + 128], w) for i in range(0, 768, 128)])  # 128 rows each
    kernels.device_check()
    assert torch.equal(pair, single)
