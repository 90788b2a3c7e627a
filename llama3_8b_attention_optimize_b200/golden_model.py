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
``get_layer0_weight_paths`` :59-93 (index.json shard map / single file)  host (no network)
``load_layer0_weights``  :96-121                                      safetensors read
``main``                 :201-249 (load, seeded input, run, dump)     all of the above
=======================  ===========================================  ==========================

With ``debug=True`` (the default, the reference's behaviour) every stage is
produced by its own bit-exact kernel, S x S tensors included.  With
``debug=False`` the attention core runs as the fused tcgen05 kernel and the
S x S stages are omitted from the dump.
"""
from __future__ import annotations

import json
import os

import numpy as np
import torch

from . import kernels

MODEL_REPO = "NousResearch/Meta-Llama-3-8B"
LOCAL_SAFETENSORS_DIR = "../llama3_weights"
OUTPUT_DIR = "./golden_model_outputs"
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


def _layer_weight_names(layer: int) -> list:
    return [f"model.layers.{layer}.self_attn.{n}_proj.weight" for n in ("q", "k", "v", "o")]


def get_layer0_weight_paths(local_dir: str | None = LOCAL_SAFETENSORS_DIR, layer: int = LAYER_IDX) -> dict:
    """Tensor name -> safetensors file for the layer's q/k/v/o_proj weights (reference
    :59-93).  A local directory with ``model.safetensors.index.json`` is resolved through
    its weight map, otherwise ``model.safetensors`` in it holds everything; with no local
    directory the files come from the Hugging Face cache / hub (``MODEL_REPO``), which
    needs network access or a populated cache."""
    names = _layer_weight_names(layer)
    if local_dir is not None and os.path.isdir(local_dir):
        index_path = os.path.join(local_dir, "model.safetensors.index.json")
        if os.path.exists(index_path):
            with open(index_path, "r") as f:
                weight_map = json.load(f)["weight_map"]
            missing = [n for n in names if n not in weight_map]
            if missing:
                raise KeyError(f"{index_path}: no entry for {missing}")
            return {n: os.path.join(local_dir, weight_map[n]) for n in names}
        return {n: os.path.join(local_dir, "model.safetensors") for n in names}
    from huggingface_hub import hf_hub_download

    with open(hf_hub_download(repo_id=MODEL_REPO, filename="model.safetensors.index.json"), "r") as f:
        weight_map = json.load(f)["weight_map"]
    shards: dict = {}
    out = {}
    for n in names:
        shard = weight_map[n]
        if shard not in shards:
            shards[shard] = hf_hub_download(repo_id=MODEL_REPO, filename=shard)
        out[n] = shards[shard]
    return out


def load_layer0_weights(local_dir: str | None = LOCAL_SAFETENSORS_DIR, layer: int = LAYER_IDX):
    """(q_proj, k_proj, v_proj, o_proj) as fp32 CPU tensors holding bf16 values, HF
    [out, in] layout (reference :96-121)."""
    from safetensors import safe_open

    paths = get_layer0_weight_paths(local_dir, layer)
    opened = {}
    weights = {}
    for name, path in paths.items():
        if path not in opened:
            opened[path] = safe_open(path, framework="pt")
        if name not in opened[path].keys():
            raise KeyError(f"{path}: tensor {name} not found")
        weights[name] = opened[path].get_tensor(name)
    return tuple(to_bf16(weights[n].float()) for n in _layer_weight_names(layer))


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


def main(local_dir: str | None = LOCAL_SAFETENSORS_DIR, output_dir: str = OUTPUT_DIR, seq_len: int = SEQ_LEN,
         device=None) -> dict:
    """The reference's main() (:201-249) on the B200: load layer-0 weights, draw the
    seeded bf16 input (torch.manual_seed(42), N(0, 0.02^2) [seq_len, 4096]), run every
    stage and write full/ and fpga_slice/ dumps (weights and input included).  Returns
    the dump."""
    q_proj, k_proj, v_proj, o_proj = load_layer0_weights(local_dir)
    torch.manual_seed(42)
    hidden_states = to_bf16(torch.randn(seq_len, HIDDEN_SIZE) * 0.02)
    if device is not None:
        dev = torch.device(device)
        hidden_states, q_proj, k_proj, v_proj, o_proj = (t.to(dev) for t in
                                                         (hidden_states, q_proj, k_proj, v_proj, o_proj))
    dump = run_full_attention(hidden_states, q_proj, k_proj, v_proj, o_proj)
    save_dump(dump, output_dir, weights={"hidden_states_input": hidden_states, "q_proj": q_proj,
                                         "k_proj": k_proj, "v_proj": v_proj, "o_proj": o_proj})
    return dump
