"""Drop-in for the reference's golden model, computed on the B200.

Same names, argument meaning and return values as llama3_attention_golden_model.py
of the reference (xuanhaozhang883/Llama3-8B-Attention-Optimize); tensors may be
given on the CPU (as the reference does) or on a CUDA device, and results come
back on the input's device as fp32 tensors holding bf16-exact values.

=======================  ===========================================  ==========================
function                 reference                                    computed by
=======================  ===========================================  ==========================
``to_bf16``              :44-47                                       dtype round trip
``save_bf16_npy``        :50-54                                       host write
``build_rope_cache``     :124-130                                     gqa_rope_cache_bf16
``rotate_half``          :133-135                                     torch (index shuffle)
``apply_rope``           :138-139 (+ the to_bf16 at :163-164)         gqa_rope_bf16
``run_full_attention``   :144-197 (all stage dumps)                   tcgen05 GEMMs + stage kernels
``run_attention_core``   :157-190 without the projections             stage kernels / fused kernel
``save_dump``            :214-246 (full/ and fpga_slice/ .npy files)  host write
=======================  ===========================================  ==========================

With ``debug=True`` (the default, the reference's behaviour) every stage is
produced by its own bit-exact kernel, S x S tensors included.  With
``debug=False`` the attention core runs as the fused tcgen05 kernel and the
S x S stages are omitted from the dump.
"""
from __future__ import annotations

import os

import numpy as np
import torch

from . import kernels

LAYER_IDX = 0
SEQ_LEN = 256
HIDDEN_SIZE = 4096
NUM_Q_HEADS = 32
NUM_KV_HEADS = 8
HEAD_DIM = 128
ROPE_THETA = 500000.0
FPGA_KV_GROUP_IDX = 0
FPGA_SEQ_LEN = 128

STAGE_NAMES = ("q_before_rope", "k_before_rope", "v", "q_after_rope", "k_after_rope", "scores_before_mask",
               "scores_after_mask", "softmax_weights", "attn_out_per_head", "final_output")


def _dev(device=None) -> torch.device:
    if device is not None:
        return torch.device(device)
    if not torch.cuda.is_available():
        raise RuntimeError("a CUDA (sm_100a) device is required; there is no CPU path")
    return torch.device("cuda", torch.cuda.current_device())


def _to_gpu_bf16(x: torch.Tensor, device: torch.device) -> torch.Tensor:
    return x.to(device=device, dtype=torch.bfloat16).contiguous()


def _back(x: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    return x.to(dtype=torch.float32, device=like.device)


def to_bf16(x: torch.Tensor) -> torch.Tensor:
    """Round to bf16 and return fp32 holding the rounded values (reference :44-47)."""
    return x.to(torch.bfloat16).to(torch.float32)


def save_bf16_npy(path: str, tensor: torch.Tensor) -> np.ndarray:
    """Round to bf16 and save as a float32 .npy (reference :50-54)."""
    arr = to_bf16(tensor).detach().cpu().numpy()
    np.save(path, arr)
    return arr


def build_rope_cache(seq_len: int, head_dim: int, theta: float, device=None):
    """(cos, sin) [seq_len, head_dim] fp32 holding bf16 values (reference :124-130)."""
    dev = _dev(device)
    cos, sin = kernels.rope_cache(seq_len, head_dim, theta, device=dev)
    out_dev = torch.device("cpu") if device is None else dev
    return cos.to(torch.float32).to(out_dev), sin.to(torch.float32).to(out_dev)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """cat(-x[..., d/2:], x[..., :d/2]) (reference :133-135)."""
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([-x2, x1], dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """bf16(x*cos + rotate_half(x)*sin) for x [H, S, d] (reference :138-139 followed by
    its to_bf16 at :163-164; inputs must hold bf16 values as in the reference)."""
    dev = x.device if x.is_cuda else _dev()
    y = kernels.rope(_to_gpu_bf16(x, dev), _to_gpu_bf16(cos, dev), _to_gpu_bf16(sin, dev))
    return _back(y, x)


def run_attention_core(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = True,
                       debug: bool = True, theta: float = ROPE_THETA) -> dict:
    """Stages q/k RoPE -> scores -> mask -> softmax -> PV for q [Hq,S,d], k/v [Hkv,S,d]
    (pre-RoPE, bf16 values).  Returns the reference's dump dict (:157-190)."""
    dev = q.device if q.is_cuda else _dev()
    qg, kg, vg = (_to_gpu_bf16(t, dev) for t in (q, k, v))
    S, d = qg.shape[-2], qg.shape[-1]
    cos, sin = kernels.rope_cache(S, d, theta, device=dev)
    dump = {"q_before_rope": qg, "k_before_rope": kg, "v": vg}
    if debug:
        qr = kernels.rope(qg, cos, sin)
        kr = kernels.rope(kg, cos, sin)
        sc = kernels.scores(qr, kr)
        sm = kernels.mask(sc, causal)
        w = kernels.softmax(sm)
        out = kernels.pv(w, vg)
        dump.update(q_after_rope=qr, k_after_rope=kr, scores_before_mask=sc, scores_after_mask=sm,
                    softmax_weights=w, attn_out_per_head=out)
    else:
        dump.update(q_after_rope=kernels.rope(qg, cos, sin), k_after_rope=kernels.rope(kg, cos, sin))
        dump["attn_out_per_head"] = kernels.prefill(qg, kg, vg, cos, sin, causal=causal, rope_q=True, rope_k=True)
    return {key: _back(val, q) for key, val in dump.items()}


def run_full_attention(hidden_states: torch.Tensor, q_proj: torch.Tensor, k_proj: torch.Tensor,
                       v_proj: torch.Tensor, o_proj: torch.Tensor, *, debug: bool = True) -> dict:
    """Full attention layer with every stage dump (reference :144-197).

    hidden_states [S, 4096]; q_proj [4096,4096], k_proj/v_proj [1024,4096],
    o_proj [4096,4096] (HF [out, in] layout), all bf16 values.  The projections are
    the tcgen05 GEMM: one fused launch writes q/k/v head-major (:149-155) and o_proj
    reads the head-major attention output directly (:193-194).
    """
    dev = hidden_states.device if hidden_states.is_cuda else _dev()
    h = _to_gpu_bf16(hidden_states, dev)
    wq, wk, wv, wo = (_to_gpu_bf16(w, dev) for w in (q_proj, k_proj, v_proj, o_proj))
    q, k, v = kernels.qkv_proj(h, wq, wk, wv, head_dim=HEAD_DIM)
    dump = run_attention_core(q, k, v, debug=debug)
    attn = dump["attn_out_per_head"].to(device=dev, dtype=torch.bfloat16).contiguous()
    dump["final_output"] = kernels.o_proj(attn, wo)
    return {key: _back(val, hidden_states) for key, val in dump.items()}


def fpga_slice(dump: dict, kv_group: int = FPGA_KV_GROUP_IDX, seq: int = FPGA_SEQ_LEN) -> dict:
    """The reference's fpga_slice cut: kv group g (4 q heads), first `seq` tokens (:225-243)."""
    g = NUM_Q_HEADS // NUM_KV_HEADS
    h0, h1 = kv_group * g, kv_group * g + g
    out = {}
    for key in ("q_before_rope", "q_after_rope", "attn_out_per_head"):
        out[key] = dump[key][h0:h1, :seq, :]
    for key in ("k_before_rope", "k_after_rope", "v"):
        out[key] = dump[key][kv_group:kv_group + 1, :seq, :]
    for key in ("scores_before_mask", "scores_after_mask", "softmax_weights"):
        if key in dump:
            out[key] = dump[key][h0:h1, :seq, :seq]
    return out


def save_dump(dump: dict, output_dir: str = "./golden_model_outputs", weights: dict | None = None) -> None:
    """Write full/<stage>.npy and fpga_slice/<stage>.npy like the reference's main() (:214-246)."""
    full_dir = os.path.join(output_dir, "full")
    os.makedirs(full_dir, exist_ok=True)
    for key, t in dump.items():
        save_bf16_npy(os.path.join(full_dir, f"{key}.npy"), t)
    for key, t in (weights or {}).items():
        save_bf16_npy(os.path.join(full_dir, f"{key}.npy"), t)
    fdir = os.path.join(output_dir, "fpga_slice")
    os.makedirs(fdir, exist_ok=True)
    for key, t in fpga_slice(dump).items():
        np.save(os.path.join(fdir, f"{key}.npy"), t.detach().cpu().numpy())
