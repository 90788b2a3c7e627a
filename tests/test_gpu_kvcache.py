"""GPU tests of the paged K/V cache path: RoPE-on-append (bit-exact against the oracle's
golden RoPE), decode over pages (bit-identical to the contiguous-cache decode over the
same rows, and within the decode tolerance of exact attention), the PagedKVCache
allocator, and the device-side input checks (reported, never faulting)."""
import numpy as np
import pytest
import torch

from llama3_8b_attention_optimize_b200 import _lib, kernels
from llama3_8b_attention_optimize_b200.session import PagedKVCache
from oracle import golden as g
from tests._util import bf16_ulp_of, bf16_words, randn_bf16

pytestmark = pytest.mark.gpu


def _paginate(kc: torch.Tensor, page_size: int, seed: int, spare: int = 3):
    """Scatter a contiguous cache [B,Hkv,L,128] into shuffled pages; returns (pages, table)."""
    B, Hkv, L, d = kc.shape
    n_lp = (L + page_size - 1) // page_size
    num_pages = B * n_lp + spare
    perm = np.random.default_rng(seed).permutation(num_pages)[: B * n_lp].reshape(B, n_lp)
    pages = randn_bf16((num_pages, Hkv, page_size, d), seed + 1000)  # unrelated rows everywhere else
    for b in range(B):
        for lp in range(n_lp):
            rows = kc[b, :, lp * page_size : min(L, (lp + 1) * page_size)]
            pages[int(perm[b, lp]), :, : rows.shape[1]] = rows
    return pages, torch.from_numpy(perm.astype(np.int32)).cuda()


@pytest.mark.parametrize("page_size,split", [(128, 0), (256, 512), (128, 128), (384, 0)])
def test_paged_decode_equals_contiguous(page_size, split):
    B, Hq, Hkv, L = 3, 32, 8, 1000
    q = randn_bf16((B, Hq, 128), 61)
    kc = randn_bf16((B, Hkv, L, 128), 62)
    vc = randn_bf16((B, Hkv, L, 128), 63)
    lens = torch.tensor([1000, 129, 1], dtype=torch.int32, device="cuda")
    cos, sin = kernels.rope_cache(1200)
    kp, table = _paginate(kc, page_size, 7)
    vp, _ = _paginate(vc, page_size, 7)
    ref = kernels.decode(q, kc, vc, lens, q_pos=lens, cos=cos, sin=sin, split_len=split)
    got = kernels.decode_paged(q, kp, vp, table, lens, q_pos=lens, cos=cos, sin=sin, split_len=split)
    kernels.device_check()
    assert torch.equal(got, ref)


def test_paged_decode_against_exact_attention():
    B, Hq, Hkv, L = 2, 32, 8, 700
    q = randn_bf16((B, Hq, 128), 71)
    kc = randn_bf16((B, Hkv, L, 128), 72)
    vc = randn_bf16((B, Hkv, L, 128), 73)
    lens_np = np.array([700, 300], dtype=np.int32)
    kp, table = _paginate(kc, 128, 9)
    vp, _ = _paginate(vc, 128, 9)
    out = kernels.decode_paged(q, kp, vp, table, torch.from_numpy(lens_np).cuda())
    kernels.device_check()
    qw, kw, vw = bf16_words(q), bf16_words(kc), bf16_words(vc)
    for b in range(B):
        L_b = int(lens_np[b])
        for h in range(Hq):
            ref = g.attention_rows(qw[b, h][None, None], kw[b, h // 4 : h // 4 + 1, :L_b],
                                   vw[b, h // 4 : h // 4 + 1, :L_b], [0], [0], causal=False)[0]
            got = g.bf16_words_to_f32(bf16_words(out[b, h]))
            assert np.all(np.abs(got - ref) <= np.maximum(1e-2, bf16_ulp_of(ref)))


def test_append_contiguous_rope_bit_exact():
    B, Hkv, Lmax, n = 3, 8, 300, 5
    kc0 = randn_bf16((B, Hkv, Lmax, 128), 81)
    vc0 = randn_bf16((B, Hkv, Lmax, 128), 82)
    kn = randn_bf16((B, Hkv, n, 128), 83)
    vn = randn_bf16((B, Hkv, n, 128), 84)
    lens_np = np.array([0, 17, Lmax - n], dtype=np.int32)
    lens = torch.from_numpy(lens_np).cuda()
    cos, sin = kernels.rope_cache(Lmax)
    kc, vc = kc0.clone(), vc0.clone()
    lens_out = torch.zeros_like(lens)
    kernels.kv_append(kn, vn, kc, vc, lens, cos=cos, sin=sin, lens_out=lens_out)
    kernels.device_check()
    assert lens_out.tolist() == (lens_np + n).tolist()
    oc, osn = g.rope_table(Lmax)
    knw = bf16_words(kn)
    for b in range(B):
        p0 = int(lens_np[b])
        ref = g.rope_apply(knw[b], oc[p0 : p0 + n], osn[p0 : p0 + n])
        assert np.array_equal(bf16_words(kc[b, :, p0 : p0 + n]), ref)
        assert torch.equal(vc[b, :, p0 : p0 + n], vn[b])
        keep = torch.ones(Lmax, dtype=torch.bool)
        keep[p0 : p0 + n] = False
        assert torch.equal(kc[b][:, keep], kc0[b][:, keep]) and torch.equal(vc[b][:, keep], vc0[b][:, keep])
    # lens_out may be lens itself; without tables K is copied unrotated (lens still
    # holds the old positions: the first call wrote the advanced lengths elsewhere)
    kernels.kv_append(kn, vn, kc, vc, lens, lens_out=lens)
    kernels.device_check()
    assert lens.tolist() == (lens_np + n).tolist()
    assert torch.equal(kc[1, :, 17:22], kn[1])


@pytest.mark.parametrize("page_size", [16, 128])
def test_append_paged_equals_contiguous(page_size):
    B, Hkv, n = 2, 8, 40
    cap_pages = 4
    Lmax = cap_pages * page_size
    kn = randn_bf16((B, Hkv, n, 128), 91)
    vn = randn_bf16((B, Hkv, n, 128), 92)
    lens = torch.tensor([3, Lmax - n], dtype=torch.int32, device="cuda")
    cos, sin = kernels.rope_cache(Lmax)
    kc = torch.zeros(B, Hkv, Lmax, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    kernels.kv_append(kn, vn, kc, vc, lens, cos=cos, sin=sin)
    kp, table = _paginate(torch.zeros_like(kc), page_size, 5)
    vp = kp.clone()
    kernels.kv_append(kn, vn, kp, vp, lens, cos=cos, sin=sin, block_table=table)
    kernels.device_check()
    for b in range(B):
        for lp in range(cap_pages):
            pg = int(table[b, lp])
            assert torch.equal(kp[pg], kc[b, :, lp * page_size : (lp + 1) * page_size])
            assert torch.equal(vp[pg], vc[b, :, lp * page_size : (lp + 1) * page_size])


def test_paged_cache_serving_loop_matches_full_prompt():
    """Prompt appended in chunks then token by token; every decode equals the contiguous
    decode over K rotated in one pass (the golden model's whole-prompt RoPE)."""
    B, Hq, Hkv = 2, 32, 8
    steps = [300, 1, 1, 130, 1]
    total = sum(steps)
    cache = PagedKVCache(B, num_pages=12, max_pages_per_seq=4, Hkv=Hkv, Hq=Hq, page_size=128)
    k_all = randn_bf16((B, Hkv, total, 128), 101)
    v_all = randn_bf16((B, Hkv, total, 128), 102)
    q_all = randn_bf16((len(steps), B, Hq, 128), 103)
    cos, sin = kernels.rope_cache(total + 1)
    k_rot = kernels.rope(k_all.view(B * Hkv, total, 128).contiguous(), cos, sin).view(B, Hkv, total, 128)
    done = 0
    for t, n in enumerate(steps):
        cache.append(k_all[:, :, done : done + n].contiguous(), v_all[:, :, done : done + n].contiguous())
        done += n
        assert [cache.seq_len(b) for b in range(B)] == [done] * B
        q_pos = torch.full((B,), done - 1, dtype=torch.int32, device="cuda")
        got = cache.decode(q_all[t], q_pos)
        lens = torch.full((B,), done, dtype=torch.int32, device="cuda")
        ref = kernels.decode(q_all[t], k_rot[:, :, :done].contiguous(), v_all[:, :, :done].contiguous(), lens,
                             q_pos=q_pos, cos=cos, sin=sin)
        kernels.device_check()
        assert torch.equal(got, ref), t
    assert cache.free_pages == 12 - 2 * 4
    cache.release(0)
    assert cache.free_pages == 12 - 4 and cache.seq_len(0) == 0
    with pytest.raises(ValueError):
        cache.reserve(4 * 128 - total + 1)


def test_device_input_checks_are_reported():
    B, Hq, Hkv = 1, 32, 8
    q = randn_bf16((B, Hq, 128), 111)
    kp = randn_bf16((4, Hkv, 128, 128), 112)
    vp = randn_bf16((4, Hkv, 128, 128), 113)
    table = torch.tensor([[0, 9]], dtype=torch.int32, device="cuda")  # page 9 is outside the pool
    lens = torch.tensor([200], dtype=torch.int32, device="cuda")
    kernels.decode_paged(q, kp, vp, table, lens)
    with pytest.raises(_lib.GqaError) as ei:
        kernels.device_check()
    assert ei.value.code == _lib.GQA_ERR_DEVICE_INPUT
    kernels.device_check()  # the check cleared it
    # appending past the cache capacity skips the rows and reports it
    kn = randn_bf16((B, Hkv, 4, 128), 114)
    good = torch.tensor([[0, 1]], dtype=torch.int32, device="cuda")
    before = kp.clone()
    kernels.kv_append(kn, kn, kp, vp, torch.tensor([254], dtype=torch.int32, device="cuda"), block_table=good)
    with pytest.raises(_lib.GqaError) as ei:
        kernels.device_check()
    assert ei.value.code == _lib.GQA_ERR_DEVICE_INPUT
    assert torch.equal(kp[1, :, 126:128], kn[0, :, :2])  # the two rows that fit were written
    assert torch.equal(kp[0], before[0]) and torch.equal(kp[2:], before[2:])
