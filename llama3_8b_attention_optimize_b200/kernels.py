"""Torch-facing wrappers over the C ABI (one function per entry point).

All tensors are CUDA bf16, contiguous; calls are enqueued on the current torch
stream.  Shapes follow the reference's golden model: per-head [H][S][d], with an
optional leading batch axis.  Raises ``GqaError`` on any non-zero status.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import GQA_FLAG_CAUSAL, GQA_FLAG_ROPE_K, GQA_FLAG_ROPE_Q, GQA_GEMM_OUT_F32, GqaError, check

ROPE_THETA = 500000.0
HEAD_DIM = 128


def default_scale(head_dim: int = HEAD_DIM) -> float:
    """fl32(1/sqrt(d)), the golden's ``scale`` (llama3_attention_golden_model.py:175)."""
    return float(torch.tensor(1.0 / math.sqrt(head_dim), dtype=torch.float32))


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _need(t: torch.Tensor, name: str, dtype=torch.bfloat16) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the kernels have no CPU path)")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def rope_cache(seq_len: int, head_dim: int = HEAD_DIM, theta: float = ROPE_THETA, pos0: int = 0,
               device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """(cos, sin) bf16 [seq_len][head_dim] on the device (golden build_rope_cache :124-130)."""
    device = torch.device(device or "cuda")
    cos = torch.empty(seq_len, head_dim, dtype=torch.bfloat16, device=device)
    sin = torch.empty_like(cos)
    check(_lib.load().gqa_rope_cache_bf16(_ptr(cos), _ptr(sin), seq_len, head_dim, pos0, float(theta),
                                          _stream(device)), "gqa_rope_cache_bf16")
    return cos, sin


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, pos0: int = 0,
         out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(x*cos + rotate_half(x)*sin) for x [..., S, d] (golden apply_rope :133-139)."""
    _need(x, "x")
    _need(cos, "cos")
    _need(sin, "sin")
    S, d = x.shape[-2], x.shape[-1]
    if cos.shape[-1] != d or cos.shape[0] < pos0 + S:
        raise ValueError("rope table too short or wrong width")
    out = torch.empty_like(x) if out is None else out
    _need(out, "out")
    heads = x.numel() // (S * d)
    check(_lib.load().gqa_rope_bf16(_ptr(x), _ptr(out), _ptr(cos), _ptr(sin), heads, S, d, pos0, _stream(x.device)),
          "gqa_rope_bf16")
    return out


def _bhsd(x: torch.Tensor, name: str) -> torch.Tensor:
    if x.dim() == 3:
        return x.unsqueeze(0)
    if x.dim() != 4:
        raise ValueError(f"{name} must be [H,S,d] or [B,H,S,d]")
    return x


def scores(q: torch.Tensor, k: torch.Tensor, scale: float | None = None) -> torch.Tensor:
    """bf16(q k^T * scale) [B,Hq,S,S] (golden scores_before_mask :175-176)."""
    _need(q, "q")
    _need(k, "k")
    q4, k4 = _bhsd(q, "q"), _bhsd(k, "k")
    B, Hq, S, d = q4.shape
    Hkv = k4.shape[1]
    out = torch.empty(B, Hq, S, S, dtype=torch.bfloat16, device=q.device)
    check(_lib.load().gqa_scores_bf16(_ptr(q4), _ptr(k4), _ptr(out), B, Hq, Hkv, S, d,
                                      default_scale(d) if scale is None else float(scale), _stream(q.device)),
          "gqa_scores_bf16")
    return out if q.dim() == 4 else out[0]


def mask(s: torch.Tensor, causal: bool = True) -> torch.Tensor:
    """bf16(s + triu(-inf, 1)) (golden scores_after_mask :180-181)."""
    _need(s, "scores")
    S = s.shape[-1]
    out = torch.empty_like(s)
    check(_lib.load().gqa_mask_bf16(_ptr(s), _ptr(out), s.numel() // (S * S), S, int(causal), _stream(s.device)),
          "gqa_mask_bf16")
    return out


def attention_mask_words(raw: torch.Tensor, q_heads: int, seq_len: int, causal: bool = True,
                         mask_value: int = _lib.GQA_MASK_NEG_INF_BF16) -> torch.Tensor:
    """Raw-word mask of the HLS kernel (attention_mask.cpp:3-58) on int16/bf16 words."""
    if raw.dtype not in (torch.int16, torch.bfloat16, torch.uint16):
        raise TypeError("raw must hold 16-bit words")
    if not raw.is_cuda or not raw.is_contiguous():
        raise ValueError("raw must be a contiguous CUDA tensor")
    out = torch.empty_like(raw)
    check(_lib.load().gqa_attention_mask_bf16(_ptr(raw), _ptr(out), q_heads, seq_len, int(causal), mask_value,
                                              _stream(raw.device)), "gqa_attention_mask_bf16")
    return out


def softmax(s: torch.Tensor) -> torch.Tensor:
    """bf16(softmax(s, -1)) (golden softmax_weights :185)."""
    _need(s, "scores")
    out = torch.empty_like(s)
    cols = s.shape[-1]
    check(_lib.load().gqa_softmax_bf16(_ptr(s), _ptr(out), s.numel() // cols, cols, _stream(s.device)),
          "gqa_softmax_bf16")
    return out


def pv(p: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """bf16(p v) with fp32 accumulation (golden attn_out_per_head :189)."""
    _need(p, "probs")
    _need(v, "v")
    p4, v4 = _bhsd(p, "p"), _bhsd(v, "v")
    B, Hq, S, _ = p4.shape
    Hkv, d = v4.shape[1], v4.shape[3]
    out = torch.empty(B, Hq, S, d, dtype=torch.bfloat16, device=p.device)
    check(_lib.load().gqa_pv_bf16(_ptr(p4), _ptr(v4), _ptr(out), B, Hq, Hkv, S, d, _stream(p.device)), "gqa_pv_bf16")
    return out if p.dim() == 4 else out[0]


def prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor | None = None,
            sin: torch.Tensor | None = None, *, causal: bool = True, rope_q: bool = False, rope_k: bool = False,
            scale: float | None = None, kv_heads: tuple[int, int] | None = None,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused GQA attention core (tcgen05): O = softmax(mask(rope(Q) rope(K)^T * scale)) V.

    q [B,Hq,S,128], k/v [B,Hkv,S,128] (or without B); rope_q/rope_k rotate in the
    kernel with the (cos, sin) tables of ``rope_cache``.  ``kv_heads=(begin, count)``
    restricts the work to one KV-head shard; other heads of ``out`` are untouched.
    """
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _need(t, n)
    q4, k4, v4 = _bhsd(q, "q"), _bhsd(k, "k"), _bhsd(v, "v")
    B, Hq, S, d = q4.shape
    Hkv = k4.shape[1]
    if k4.shape != (B, Hkv, S, d) or v4.shape != k4.shape:
        raise ValueError("k and v must be [B,Hkv,S,d] matching q")
    flags = (GQA_FLAG_CAUSAL if causal else 0) | (GQA_FLAG_ROPE_Q if rope_q else 0) | (GQA_FLAG_ROPE_K if rope_k else 0)
    if (rope_q or rope_k):
        if cos is None or sin is None:
            raise ValueError("rope_q/rope_k need cos and sin tables")
        _need(cos, "cos")
        _need(sin, "sin")
        if cos.shape[0] < S or cos.shape[1] != d:
            raise ValueError("rope table shorter than the sequence")
    if out is None:
        out = torch.empty_like(q4)
    _need(out, "out")
    kb, kc = (0, Hkv) if kv_heads is None else kv_heads
    check(_lib.load().gqa_prefill_bf16(_ptr(q4), _ptr(k4), _ptr(v4), _ptr(out),
                                       _ptr(cos) if cos is not None else None, _ptr(sin) if sin is not None else None,
                                       B, S, Hq, Hkv, d, kb, kc, default_scale(d) if scale is None else float(scale),
                                       flags, _stream(q.device)), "gqa_prefill_bf16")
    return out if q.dim() == 4 else out[0]


def decode_workspace_bytes(B: int, Hq: int, max_len: int, split_len: int = 0) -> int:
    return int(_lib.load().gqa_decode_workspace_size(B, Hq, max_len, split_len))


def decode(q: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor, lens: torch.Tensor, *,
           q_pos: torch.Tensor | None = None, cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
           workspace: torch.Tensor | None = None, split_len: int = 0, scale: float | None = None,
           kv_heads: tuple[int, int] | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Split-KV decode: q [B,Hq,128] against kcache/vcache [B,Hkv,Lmax,128]; lens int32 [B].

    With ``q_pos`` (int32 [B]) and (cos, sin), q is rotated at q_pos[b] in the kernel.
    """
    for t, n in ((q, "q"), (kcache, "kcache"), (vcache, "vcache")):
        _need(t, n)
    _need(lens, "lens", torch.int32)
    B, Hq, d = q.shape
    Hkv, Lmax = kcache.shape[1], kcache.shape[2]
    if kcache.shape != (B, Hkv, Lmax, d) or vcache.shape != kcache.shape or lens.shape != (B,):
        raise ValueError("bad decode shapes")
    flags = 0
    if q_pos is not None:
        _need(q_pos, "q_pos", torch.int32)
        _need(cos, "cos")
        _need(sin, "sin")
        if cos.shape[0] < Lmax + 1 or sin.shape[0] < Lmax + 1:
            raise ValueError("decode rope tables need max_len + 1 rows")
        flags |= GQA_FLAG_ROPE_Q
    need = decode_workspace_bytes(B, Hq, Lmax, split_len)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q) if out is None else out
    kb, kc = (0, Hkv) if kv_heads is None else kv_heads
    check(_lib.load().gqa_decode_bf16(_ptr(q), _ptr(kcache), _ptr(vcache), _ptr(lens),
                                      _ptr(q_pos) if q_pos is not None else None,
                                      _ptr(cos) if cos is not None else None, _ptr(sin) if sin is not None else None,
                                      _ptr(out), _ptr(workspace), workspace.numel() * workspace.element_size(),
                                      B, Lmax, Hq, Hkv, d, kb, kc, split_len,
                                      default_scale(d) if scale is None else float(scale), flags, _stream(q.device)),
          "gqa_decode_bf16")
    return out


def kv_append(k_new: torch.Tensor, v_new: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor,
              lens: torch.Tensor, *, cos: torch.Tensor | None = None, sin: torch.Tensor | None = None,
              block_table: torch.Tensor | None = None, lens_out: torch.Tensor | None = None) -> None:
    """Write k_new/v_new [B,Hkv,n,128] at positions lens[b] + i of the cache, K rotated
    there when (cos, sin) are given.  Contiguous cache [B,Hkv,Lmax,128], or (with
    ``block_table`` int32 [B,max_pages]) page pools [num_pages,Hkv,page_size,128].
    ``lens_out`` (may be ``lens``) receives lens + n after the writes."""
    for t, n in ((k_new, "k_new"), (v_new, "v_new"), (kcache, "kcache"), (vcache, "vcache")):
        _need(t, n)
    _need(lens, "lens", torch.int32)
    B, Hkv, n, d = k_new.shape
    if v_new.shape != k_new.shape or vcache.shape != kcache.shape or lens.shape != (B,):
        raise ValueError("bad kv_append shapes")
    flags = 0
    if cos is not None or sin is not None:
        _need(cos, "cos")
        _need(sin, "sin")
        flags |= GQA_FLAG_ROPE_K
    if block_table is not None:
        _need(block_table, "block_table", torch.int32)
        num_pages, _, page_size, _ = kcache.shape
        max_pages, max_len = block_table.shape[1], 0
        if block_table.shape[0] != B or kcache.shape[1] != Hkv:
            raise ValueError("bad paged kv_append shapes")
    else:
        if kcache.shape[:2] != (B, Hkv):
            raise ValueError("bad kv_append cache shape")
        num_pages = page_size = max_pages = 0
        max_len = kcache.shape[2]
    if lens_out is not None:
        _need(lens_out, "lens_out", torch.int32)
    capacity = max_pages * page_size if block_table is not None else max_len
    if flags and (cos.shape[0] < capacity or sin.shape[0] < capacity):
        raise ValueError("kv_append rope tables need one row per cache position")
    check(_lib.load().gqa_kv_append_bf16(_ptr(k_new), _ptr(v_new), _ptr(kcache), _ptr(vcache),
                                         _ptr(block_table) if block_table is not None else None, max_pages, page_size,
                                         num_pages, _ptr(lens), _ptr(lens_out) if lens_out is not None else None,
                                         _ptr(cos) if cos is not None else None, _ptr(sin) if sin is not None else None,
                                         B, Hkv, n, d, max_len, flags, _stream(k_new.device)), "gqa_kv_append_bf16")


def decode_paged(q: torch.Tensor, kpages: torch.Tensor, vpages: torch.Tensor, block_table: torch.Tensor,
                 lens: torch.Tensor, *, q_pos: torch.Tensor | None = None, cos: torch.Tensor | None = None,
                 sin: torch.Tensor | None = None, workspace: torch.Tensor | None = None, split_len: int = 0,
                 scale: float | None = None, kv_heads: tuple[int, int] | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Split-KV decode over page pools kpages/vpages [num_pages,Hkv,page_size,128] with
    block_table int32 [B,max_pages] (page_size a multiple of 128)."""
    for t, n in ((q, "q"), (kpages, "kpages"), (vpages, "vpages")):
        _need(t, n)
    _need(lens, "lens", torch.int32)
    _need(block_table, "block_table", torch.int32)
    B, Hq, d = q.shape
    num_pages, Hkv, page_size, _ = kpages.shape
    max_pages = block_table.shape[1]
    if vpages.shape != kpages.shape or block_table.shape[0] != B or lens.shape != (B,):
        raise ValueError("bad paged decode shapes")
    capacity = max_pages * page_size
    flags = 0
    if q_pos is not None:
        _need(q_pos, "q_pos", torch.int32)
        _need(cos, "cos")
        _need(sin, "sin")
        if cos.shape[0] < capacity + 1 or sin.shape[0] < capacity + 1:
            raise ValueError("decode rope tables need capacity + 1 rows")
        flags |= GQA_FLAG_ROPE_Q
    need = decode_workspace_bytes(B, Hq, capacity, split_len)
    if workspace is None:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q) if out is None else out
    kb, kc = (0, Hkv) if kv_heads is None else kv_heads
    check(_lib.load().gqa_decode_paged_bf16(_ptr(q), _ptr(kpages), _ptr(vpages), _ptr(block_table), max_pages,
                                            page_size, num_pages, _ptr(lens),
                                            _ptr(q_pos) if q_pos is not None else None,
                                            _ptr(cos) if cos is not None else None,
                                            _ptr(sin) if sin is not None else None, _ptr(out), _ptr(workspace),
                                            workspace.numel() * workspace.element_size(), B, Hq, Hkv, d, kb, kc,
                                            split_len, default_scale(d) if scale is None else float(scale), flags,
                                            _stream(q.device)), "gqa_decode_paged_bf16")
    return out


def linear(x: torch.Tensor, w: torch.Tensor, *, out_f32: bool = False,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(x @ w^T) (or the fp32 sums with ``out_f32``) for x [..., K], w [N, K] in the
    HF [out, in] layout (golden projections, llama3_attention_golden_model.py:149-151, :194)."""
    _need(x, "x")
    _need(w, "w")
    K = x.shape[-1]
    if w.dim() != 2 or w.shape[1] != K:
        raise ValueError("w must be [N, K] with K = x.shape[-1]")
    N, M = w.shape[0], x.numel() // K
    odt = torch.float32 if out_f32 else torch.bfloat16
    out = torch.empty(*x.shape[:-1], N, dtype=odt, device=x.device) if out is None else out
    _need(out, "out", odt)
    if out.numel() != M * N:
        raise ValueError("out has the wrong size")
    check(_lib.load().gqa_gemm_bf16(_ptr(x), _ptr(w), _ptr(out), M, N, K, K, K, N,
                                    GQA_GEMM_OUT_F32 if out_f32 else 0, _stream(x.device)), "gqa_gemm_bf16")
    return out


def qkv_proj(h: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor,
             cos: torch.Tensor | None = None, sin: torch.Tensor | None = None, *, rope_q: bool = False,
             rope_k: bool = False, pos0: int = 0, head_dim: int = HEAD_DIM,
             out: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None):
    """Fused q/k/v projection (one launch): h [S, hidden] or [B, S, hidden] -> head-major
    q [B?, Hq, S, 128], k/v [B?, Hkv, S, 128] = bf16(h @ W^T) viewed per head
    (golden :149-155); q / k rotated at positions pos0 + s when rope_q / rope_k (:162-164)."""
    for t, n in ((h, "h"), (wq, "wq"), (wk, "wk"), (wv, "wv")):
        _need(t, n)
    batched = h.dim() == 3
    B, S, hidden = (h.shape if batched else (1, *h.shape))
    Hq, Hkv = wq.shape[0] // head_dim, wk.shape[0] // head_dim
    if wq.shape != (Hq * head_dim, hidden) or wk.shape != (Hkv * head_dim, hidden) or wv.shape != wk.shape:
        raise ValueError("weights must be [H*head_dim, hidden]")
    lead = (B,) if batched else ()
    if out is None:
        q = torch.empty(*lead, Hq, S, head_dim, dtype=torch.bfloat16, device=h.device)
        k = torch.empty(*lead, Hkv, S, head_dim, dtype=torch.bfloat16, device=h.device)
        v = torch.empty_like(k)
    else:
        q, k, v = out
    flags = (GQA_FLAG_ROPE_Q if rope_q else 0) | (GQA_FLAG_ROPE_K if rope_k else 0)
    if flags:
        if cos is None or sin is None:
            raise ValueError("rope needs cos/sin tables")
        _need(cos, "cos")
        _need(sin, "sin")
        if cos.shape[0] < pos0 + S:
            raise ValueError("rope table too short")
    cp = _ptr(cos) if flags else None
    sp = _ptr(sin) if flags else None
    check(_lib.load().gqa_qkv_proj_bf16(_ptr(h), _ptr(wq), _ptr(wk), _ptr(wv), _ptr(q), _ptr(k), _ptr(v), cp, sp,
                                        B, S, hidden, Hq, Hkv, head_dim, pos0, flags, _stream(h.device)),
          "gqa_qkv_proj_bf16")
    return q, k, v


def o_proj(attn: torch.Tensor, wo: torch.Tensor, *, head_begin: int = 0, out_f32: bool = False,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """o_proj straight from the head-major attention output attn [B?, H, S, 128]:
    out [B?, S, N] = concat_h(attn) @ wo[:, head_begin*128 : (head_begin+H)*128]^T (golden :193-194)."""
    _need(attn, "attn")
    _need(wo, "wo")
    a4 = _bhsd(attn, "attn")
    B, H, S, d = a4.shape
    N, width = wo.shape
    if (head_begin + H) * d > width:
        raise ValueError("wo has fewer input columns than the heads need")
    odt = torch.float32 if out_f32 else torch.bfloat16
    shape = (B, S, N) if attn.dim() == 4 else (S, N)
    out = torch.empty(shape, dtype=odt, device=attn.device) if out is None else out
    _need(out, "out", odt)
    w_ptr = _ptr(wo) + head_begin * d * wo.element_size()
    check(_lib.load().gqa_o_proj_bf16(_ptr(attn), w_ptr, _ptr(out), B, S, H, d, N, width,
                                      GQA_GEMM_OUT_F32 if out_f32 else 0, _stream(attn.device)), "gqa_o_proj_bf16")
    return out


def o_proj_rows(attn: torch.Tensor, wo: torch.Tensor, out: torch.Tensor, s0: int, s_count: int, *,
                head_begin: int = 0, out_f32: bool = False, max_ctas: int = 0) -> torch.Tensor:
    """Rows [s0, s0+s_count) of ``o_proj`` for one sequence: attn [H, S, 128] (or
    [1, H, S, 128]) into the full-size ``out`` [S, N] (or [1, S, N]); the other rows are
    left alone.  ``max_ctas`` > 0 caps the GEMM's persistent grid."""
    _need(attn, "attn")
    _need(wo, "wo")
    a4 = _bhsd(attn, "attn")
    B, H, S, d = a4.shape
    if B != 1:
        raise ValueError("o_proj_rows takes one sequence")
    N, width = wo.shape
    if (head_begin + H) * d > width:
        raise ValueError("wo has fewer input columns than the heads need")
    odt = torch.float32 if out_f32 else torch.bfloat16
    _need(out, "out", odt)
    if out.numel() != S * N:
        raise ValueError("out must hold all S x N rows")
    w_ptr = _ptr(wo) + head_begin * d * wo.element_size()
    check(_lib.load().gqa_o_proj_rows_bf16(_ptr(attn), w_ptr, _ptr(out), S, s0, s_count, H, d, N, width, max_ctas,
                                           GQA_GEMM_OUT_F32 if out_f32 else 0, _stream(attn.device)),
          "gqa_o_proj_rows_bf16")
    return out


def cast_bf16(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Round an fp32 tensor to bf16 (RNE), e.g. all-reduced o_proj partials."""
    _need(x, "x", torch.float32)
    out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device) if out is None else out
    _need(out, "out")
    check(_lib.load().gqa_cast_f32_bf16(_ptr(x), _ptr(out), x.numel(), _stream(x.device)), "gqa_cast_f32_bf16")
    return out


def device_check(device=None) -> None:
    """Synchronize and raise if any kernel's bounded wait expired since the last check."""
    device = torch.device(device or "cuda")
    site = ctypes_int()
    rc = _lib.load().gqa_device_check(_stream(device), site)
    if rc != 0:
        raise GqaError(rc, f"device check (site 0x{site.value:x})")


def ctypes_int():
    import ctypes
    return ctypes.c_int(0)


__all__ = ["rope_cache", "rope", "scores", "mask", "attention_mask_words", "softmax", "pv", "prefill", "decode",
           "decode_workspace_bytes", "device_check", "default_scale", "GqaError"]
