"""Shared helpers for the test suite (seeded inputs, bf16 word views, ulp metrics)."""
from __future__ import annotations

import json
import os

import numpy as np
import torch

from oracle import golden as g


def bf16_words(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor (any device) -> uint16 numpy words."""
    return t.detach().to("cpu").contiguous().view(torch.int16).numpy().view(np.uint16)


def words_to_bf16(w: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(w, np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def randn_bf16(shape, seed: int, scale: float = 1.0, device="cuda") -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=gen, dtype=torch.float32) * scale
    return x.to(torch.bfloat16).to(device)


def ulp_dist(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    def key(w):
        w = w.astype(np.int64)
        return np.where(w & 0x8000, 0x8000 - (w & 0x7FFF), 0x8000 + w)
    return np.abs(key(a) - key(b))


def ulp_histogram(a_words: np.ndarray, b_words: np.ndarray) -> dict:
    """Share of elements whose bf16 words are 0, 1, 2 or more ulps apart, over all
    elements and ("big_*") over those whose reference value b has |b| >= 1/4 (below that
    a tiny absolute error spans many ulps, and outputs near zero dominate the counts)."""
    d = ulp_dist(a_words, b_words)
    mag = np.abs((np.asarray(b_words, np.uint32) << 16).view(np.float32))
    big = d[mag >= 0.25]
    frac = lambda x, sel: float(sel.mean()) if x.size else 0.0  # noqa: E731
    return {"0": frac(d, d == 0), "1": frac(d, d == 1), "2": frac(d, d == 2), ">2": frac(d, d > 2),
            "max": int(d.max()) if d.size else 0,
            "big_share": float(big.size / d.size) if d.size else 0.0,
            "big_0": frac(big, big == 0), "big_1": frac(big, big == 1), "big_>1": frac(big, big > 1),
            "big_max": int(big.max()) if big.size else 0}


def rows_reference(q_rot_w, k_rot_w, v_w, heads, pos, causal=True, n_keys=None) -> np.ndarray:
    """Exact float64-accumulated attention rows from the oracle (per batch element)."""
    return g.attention_rows(q_rot_w, k_rot_w, v_w, heads, pos, causal=causal, n_keys=n_keys)


def bf16_ulp_of(x: np.ndarray) -> np.ndarray:
    """Size of one bf16 ulp at |x| (for the output-rounding allowance)."""
    ax = np.maximum(np.abs(x).astype(np.float32), np.float32(2.0 ** -126))
    e = np.floor(np.log2(ax))
    return np.exp2(e - 7).astype(np.float32)


def report_ulps(name: str, hists) -> dict:
    """Print the mean of ulp histograms (kernel output vs the correctly rounded exact
    value) under `name` and, when GQA_PARITY_REPORT names a file, append it there as a
    JSON line.  `hists` is one ulp_histogram dict or a list of them (equal weights)."""
    hists = [hists] if isinstance(hists, dict) else list(hists)
    keys = ("0", "1", "2", ">2", "big_share", "big_0", "big_1", "big_>1")
    hist = {k: sum(h[k] for h in hists) / len(hists) for k in keys}
    hist["max"] = max(h["max"] for h in hists)
    hist["big_max"] = max(h["big_max"] for h in hists)
    print(f"ulp histogram {name}: {hist}")
    path = os.environ.get("GQA_PARITY_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"check": name, "ulp": hist}) + "\n")
    return hist
