"""Host-buffer entry points: the call a user makes with Q/K/V in (pinned) host memory.

``PrefillSession`` / ``DecodeSession`` own the device buffers and RoPE tables for
one shape, so repeated calls allocate nothing; each call copies the inputs
host->device, runs the kernel and copies the result device->host on the
current stream.  This is the end-to-end path that replaces calling the
reference's ``gqa_attention_cpu`` / ``run_full_attention`` on host arrays.
"""
from __future__ import annotations

import torch

from . import kernels


ROPE_MODES = ("prepass_k", "fused", "none")


class PrefillSession:
    """Device buffers + RoPE tables for one prefill shape.

    rope = "prepass_k" (default): K is rotated once by gqa_rope_bf16 into a session
           buffer, Q is rotated on load inside the fused kernel.
    rope = "fused":     both rotated inside the fused kernel (every CTA that reads a K
           tile rotates it again; no extra buffer).
    rope = "none":      inputs already rotated.
    """

    def __init__(self, B: int, S: int, Hq: int, Hkv: int, head_dim: int = 128, *, causal: bool = True,
                 rope: str = "prepass_k", theta: float = kernels.ROPE_THETA, device=None):
        if rope not in ROPE_MODES:
            raise ValueError(f"rope must be one of {ROPE_MODES}")
        self.device = torch.device(device or "cuda")
        self.shape_q = (B, Hq, S, head_dim)
        self.shape_kv = (B, Hkv, S, head_dim)
        mk = lambda shp: torch.empty(shp, dtype=torch.bfloat16, device=self.device)  # noqa: E731
        self.q, self.k, self.v, self.o = mk(self.shape_q), mk(self.shape_kv), mk(self.shape_kv), mk(self.shape_q)
        self.k_rot = mk(self.shape_kv) if rope == "prepass_k" else None
        self.causal, self.rope = causal, rope
        self.cos, self.sin = kernels.rope_cache(S, head_dim, theta, device=self.device) if rope != "none" \
            else (None, None)

    def launches_per_step(self) -> int:
        return 2 if self.rope == "prepass_k" else 1

    def h2d_bytes(self) -> int:
        return (self.q.numel() + self.k.numel() + self.v.numel()) * 2

    def d2h_bytes(self) -> int:
        return self.o.numel() * 2

    def run_device(self) -> torch.Tensor:
        if self.rope == "prepass_k":
            kernels.rope(self.k, self.cos, self.sin, out=self.k_rot)
            return kernels.prefill(self.q, self.k_rot, self.v, self.cos, self.sin, causal=self.causal, rope_q=True,
                                   out=self.o)
        fused = self.rope == "fused"
        return kernels.prefill(self.q, self.k, self.v, self.cos, self.sin, causal=self.causal, rope_q=fused,
                               rope_k=fused, out=self.o)

    def capture(self) -> torch.cuda.CUDAGraph:
        """Record one ``run_device()`` step (K pre-pass and fused kernel) in a CUDA graph.

        ``graph.replay()`` then re-runs the step on this session's buffers with one launch
        from the host: short prompts (seq 128 .. 2048) take tens of microseconds on the GPU,
        about what launching the two kernels through Python costs.  Refill ``q``/``k``/``v``
        in place between replays.  The first step runs outside the capture, so the
        library's per-device set-up (shared-memory attributes, the register-count check)
        is done before it.
        """
        self.run_device()
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.run_device()
        return graph

    def run_host(self, q_h: torch.Tensor, k_h: torch.Tensor, v_h: torch.Tensor, out_h: torch.Tensor) -> torch.Tensor:
        """q_h/k_h/v_h/out_h: bf16 CPU tensors (pin them for asynchronous copies)."""
        self.q.copy_(q_h, non_blocking=True)
        self.k.copy_(k_h, non_blocking=True)
        self.v.copy_(v_h, non_blocking=True)
        self.run_device()
        out_h.copy_(self.o, non_blocking=True)
        return out_h


class PrefillStream:
    """Host-buffer prefill over a sequence of steps with the copies overlapped.

    Two device buffer sets and three CUDA streams: while step i computes, step i+1's
    Q/K/V go host->device and step i-1's O goes device->host, so a step costs the
    slowest of the three instead of their sum.  Every step still copies its own inputs
    in and its output out.  ``run`` enqueues everything and makes the caller's current
    stream wait for the last copy-out; synchronise (or record an event) after it.
    """

    def __init__(self, B: int, S: int, Hq: int, Hkv: int, head_dim: int = 128, *, causal: bool = True,
                 rope: str = "prepass_k", theta: float = kernels.ROPE_THETA, device=None):
        self.device = torch.device(device or "cuda")
        self.sets = [PrefillSession(B, S, Hq, Hkv, head_dim, causal=causal, rope=rope, theta=theta, device=self.device)
                     for _ in range(2)]
        self.s_in, self.s_comp, self.s_out = (torch.cuda.Stream(self.device) for _ in range(3))

    def h2d_bytes(self) -> int:
        return self.sets[0].h2d_bytes()

    def d2h_bytes(self) -> int:
        return self.sets[0].d2h_bytes()

    def launches_per_step(self) -> int:
        return self.sets[0].launches_per_step()

    def run(self, steps) -> None:
        """steps: iterable of (q_h, k_h, v_h, out_h) bf16 CPU tensors (pinned)."""
        cur = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(cur)
        for st in (self.s_in, self.s_comp, self.s_out):
            st.wait_event(start)
        ev_comp, ev_out = [], []
        last = None
        for i, (q_h, k_h, v_h, out_h) in enumerate(steps):
            sess = self.sets[i % 2]
            with torch.cuda.stream(self.s_in):
                if i >= 2:  # this buffer set's inputs were consumed by step i-2
                    self.s_in.wait_event(ev_comp[i - 2])
                sess.q.copy_(q_h, non_blocking=True)
                sess.k.copy_(k_h, non_blocking=True)
                sess.v.copy_(v_h, non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(self.s_in)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(ev_in)
                if i >= 2:  # and its output was read out by step i-2's copy
                    self.s_comp.wait_event(ev_out[i - 2])
                sess.run_device()
                e = torch.cuda.Event()
                e.record(self.s_comp)
                ev_comp.append(e)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(e)
                out_h.copy_(sess.o, non_blocking=True)
                last = torch.cuda.Event()
                last.record(self.s_out)
                ev_out.append(last)
        if last is not None:
            cur.wait_event(last)


class DecodeSession:
    def __init__(self, B: int, Lmax: int, Hq: int, Hkv: int, head_dim: int = 128, *, split_len: int = 0,
                 rope_q: bool = True, theta: float = kernels.ROPE_THETA, device=None):
        self.device = torch.device(device or "cuda")
        self.B, self.Lmax, self.Hq, self.Hkv = B, Lmax, Hq, Hkv
        self.split_len = split_len
        self.q = torch.empty(B, Hq, head_dim, dtype=torch.bfloat16, device=self.device)
        self.o = torch.empty_like(self.q)
        self.lens = torch.empty(B, dtype=torch.int32, device=self.device)
        self.ws = torch.empty(kernels.decode_workspace_bytes(B, Hq, Lmax, split_len), dtype=torch.uint8,
                              device=self.device)
        self.cos, self.sin = kernels.rope_cache(Lmax + 1, head_dim, theta, device=self.device) if rope_q else (None, None)
        self.rope_q = rope_q

    def run_device(self, kcache: torch.Tensor, vcache: torch.Tensor) -> torch.Tensor:
        return kernels.decode(self.q, kcache, vcache, self.lens, q_pos=self.lens if self.rope_q else None,
                              cos=self.cos, sin=self.sin, workspace=self.ws, split_len=self.split_len, out=self.o)

    def run_host(self, q_h: torch.Tensor, lens_h: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor,
                 out_h: torch.Tensor) -> torch.Tensor:
        """One decode step: the new tokens' q and the cache lengths come from the host;
        the KV cache stays resident on the device (as in serving)."""
        self.q.copy_(q_h, non_blocking=True)
        self.lens.copy_(lens_h, non_blocking=True)
        self.run_device(kcache, vcache)
        out_h.copy_(self.o, non_blocking=True)
        return out_h


class PagedKVCache:
    """Paged K/V cache for serving decode: page pools on the device, block tables and a
    free list of pages kept on the host.

    Pools ``k``/``v`` are [num_pages, Hkv, page_size, 128] bf16; ``table`` int32
    [B, max_pages_per_seq] maps a sequence's logical page to a pool page (-1 = none);
    ``lens`` int32 [B] on the device is the number of cached tokens per sequence.
    ``append`` reserves pages, writes the new rows with K rotated at their positions
    (``gqa_kv_append_bf16``) and advances ``lens``; ``decode`` runs the split-KV decode
    over the pages (``gqa_decode_paged_bf16``) with q rotated at its position.
    """

    def __init__(self, B: int, num_pages: int, max_pages_per_seq: int, Hkv: int = 8, Hq: int = 32,
                 page_size: int = 128, head_dim: int = 128, *, split_len: int = 0,
                 theta: float = kernels.ROPE_THETA, device=None):
        if page_size % 128:
            raise ValueError("page_size must be a multiple of 128")
        self.device = torch.device(device or "cuda")
        self.B, self.Hkv, self.Hq, self.page_size = B, Hkv, Hq, page_size
        self.max_pages = max_pages_per_seq
        self.capacity = max_pages_per_seq * page_size
        self.split_len = split_len
        shape = (num_pages, Hkv, page_size, head_dim)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.table = torch.full((B, max_pages_per_seq), -1, dtype=torch.int32, device=self.device)
        self.lens = torch.zeros(B, dtype=torch.int32, device=self.device)
        self._table_h = [[-1] * max_pages_per_seq for _ in range(B)]
        self._lens_h = [0] * B
        self._free = list(range(num_pages - 1, -1, -1))
        self.cos, self.sin = kernels.rope_cache(self.capacity + 1, head_dim, theta, device=self.device)
        self.ws = torch.empty(max(kernels.decode_workspace_bytes(B, Hq, self.capacity, split_len), 16),
                              dtype=torch.uint8, device=self.device)

    @property
    def free_pages(self) -> int:
        return len(self._free)

    def seq_len(self, b: int) -> int:
        return self._lens_h[b]

    def reserve(self, n_new: int) -> None:
        """Give every sequence pages for n_new more tokens (raises when out of pages)."""
        changed = False
        for b in range(self.B):
            need = self._lens_h[b] + n_new
            if need > self.capacity:
                raise ValueError(f"sequence {b}: {need} tokens exceed the capacity {self.capacity}")
            for lp in range((need + self.page_size - 1) // self.page_size):
                if self._table_h[b][lp] < 0:
                    if not self._free:
                        raise RuntimeError("paged KV cache: out of pages")
                    self._table_h[b][lp] = self._free.pop()
                    changed = True
        if changed:
            self.table.copy_(torch.tensor(self._table_h, dtype=torch.int32))

    def release(self, b: int) -> None:
        """Return sequence b's pages to the free list and reset its length."""
        for lp, page in enumerate(self._table_h[b]):
            if page >= 0:
                self._free.append(page)
                self._table_h[b][lp] = -1
        self._lens_h[b] = 0
        self.table[b].fill_(-1)
        self.lens[b] = 0

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """k_new/v_new [B, Hkv, n, 128] (K before RoPE): cached at positions lens[b] + i."""
        n = k_new.shape[2]
        self.reserve(n)
        kernels.kv_append(k_new, v_new, self.k, self.v, self.lens, cos=self.cos, sin=self.sin,
                          block_table=self.table, lens_out=self.lens)
        self._lens_h = [x + n for x in self._lens_h]

    def decode(self, q: torch.Tensor, q_pos: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """q [B, Hq, 128] (before RoPE) at positions q_pos (int32 [B]) over the cached tokens."""
        return kernels.decode_paged(q, self.k, self.v, self.table, self.lens, q_pos=q_pos, cos=self.cos,
                                    sin=self.sin, workspace=self.ws, split_len=self.split_len, out=out)
