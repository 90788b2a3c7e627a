"""Benchmark: fused causal GQA prefill TFLOP/s at seq 8192 (+ decode HBM GB/s) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload (one step = one launch of the fused kernel over one batch):
  causal GQA prefill, Hq=32, Hkv=8, d=128, seq 8192, bf16, from un-rotated Q/K: RoPE
  (theta 5e5) on K by one pre-pass kernel and on Q inside the fused kernel (--rope fused
  rotates both inside the fused kernel); Q,K ~ 2.5*N(0,1), V ~ N(0,1) (seeded synthetic).
  N=1: batch 4 (the headline configuration).  N GPUs: batch 4N, rank r owns kv
  heads [8r/N, 8(r+1)/N) of every sequence (KV-head sharding, no collective), so the
  work per GPU is fixed ("weak" scaling).  Inputs (335 MB per rank) exceed L2.
Also measured: split-KV decode, batch 64 (64N across ranks), cache lengths
U[1024, 32768], reported in HBM GB/s under "decode"; and one full attention layer
(seq 4096, hidden 4096: fused q/k/v projection with RoPE, causal core, o_proj, and
across ranks an fp32 NCCL all-reduce of the row-parallel o_proj partials) in TFLOP/s
under "full_layer" (total work fixed: strong scaling).

Prints ONE JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HQ, HKV, D, S_PREFILL, B_PER_GPU = 32, 8, 128, 8192, 4
LAYER_S = 4096
DEC_B, DEC_LMAX = 64, 32768
METRIC = "GQA causal prefill TFLOP/s (seq 8192) at 1/2/4/8 B200; decode HBM GB/s"


def causal_flops(B, Hq, S, d):
    return 4.0 * B * Hq * d * S * (S + 1) / 2.0


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p.get("bf16_tflops_sustained"), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def load_profile_traffic():
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f)
    except Exception:
        return {}


class ClockSampler:
    """nvidia-smi sampling of SM clocks / throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []
        self.t0, self.t1 = None, None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "20", "-i", str(self.idx)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.5)  # nvidia-smi is sampling before the timed region starts
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def window(self, t0: float, t1: float):
        """Keep only the samples taken while the timed region ran."""
        self.t0, self.t1 = t0, t1

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        rows = []
        for t, ln in self.lines:
            if self.t0 is not None and not (self.t0 <= t <= self.t1 + 0.15):
                continue
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, fl in rows for i, v in enumerate(fl) if v.lower().startswith("active")})
        loaded = [r[0] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int, device: str = "cuda") -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_loop(fn, steps, world, stream):
    """K back-to-back calls bracketed by barrier + synchronize; CUDA events on `stream`."""
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1), world)


def cpu_reference_sample(heads: int, S: int, seed: int = 7):
    """The reference's NumPy fp32 core (oracle port) on `heads` query heads of the
    workload; returns (seconds, causal flops of the sample, threads)."""
    from oracle import cpu_port
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((heads, S, D), dtype=np.float32) * np.float32(2.5))
    k = (rng.standard_normal((1, S, D), dtype=np.float32) * np.float32(2.5))
    v = rng.standard_normal((1, S, D), dtype=np.float32)
    t0 = time.perf_counter()
    for h in range(heads):
        cpu_port.gqa_attention_head(q[h], k[0], v[0], causal=True)
    dt = time.perf_counter() - t0
    return dt, causal_flops(1, heads, S, D), os.cpu_count()


# The reference's one published figure: CPU_Baseline fp32 at 32 q heads, 8 kv heads,
# seq 128, head_dim 128, median of 50 runs after 10 warm-up runs, on its author's CPU.
REFERENCE_C1_PUBLISHED_MS = 2.088770


def cpu_small_configs() -> dict:
    """The NumPy port of gqa_attention_cpu at the reference's own benchmark settings:
    seq 128 (its published configuration; warm-up 10, repeat 50, median, as its
    run_benchmark times it) and seq 2048 (warm-up 1, repeat 3), fp32, generate_qkv inputs."""
    from oracle import cpu_port

    out = {"c1_published_ms": REFERENCE_C1_PUBLISHED_MS,
           "small_configs": "CPU_Baseline llama3_like shapes (32 q / 8 kv heads, d 128), fp32, causal, "
                            "generate_qkv(seed 2026), all host threads"}
    for key, S, warm, rep in (("c1", 128, 10, 50), ("c2", 2048, 1, 3)):
        cfg = cpu_port.BaselineConfig(q_heads=HQ, kv_heads=HKV, seq_len=S, head_dim=D)
        q, k, v = cpu_port.generate_qkv(cfg)
        for _ in range(warm):
            cpu_port.gqa_attention_cpu(q, k, v, cfg)
        ts = []
        for _ in range(rep):
            t0 = time.perf_counter()
            cpu_port.gqa_attention_cpu(q, k, v, cfg)
            ts.append(time.perf_counter() - t0)
        out[f"{key}_ms"] = 1e3 * statistics.median(ts)
        out[f"{key}_repeat"] = rep
    return out


def run_short_prefills(args, hq, hkv, dev, stream, world) -> dict:
    """Batch 1 prefill at seq 128 and seq 2048 (this rank's heads), timed like the
    headline step; at these sizes launch overhead and wave quantisation dominate."""
    from llama3_8b_attention_optimize_b200 import kernels
    from llama3_8b_attention_optimize_b200.session import PrefillSession

    out = {}
    gen = torch.Generator(device=dev).manual_seed(2026)
    for key, S in (("c1", 128), ("c2", 2048)):
        sess = PrefillSession(1, S, hq, hkv, D, causal=True, rope=args.rope, device=dev)
        sess.q.copy_(torch.randn(sess.shape_q, generator=gen, device=dev))
        sess.k.copy_(torch.randn(sess.shape_kv, generator=gen, device=dev))
        sess.v.copy_(torch.randn(sess.shape_kv, generator=gen, device=dev))
        for _ in range(max(args.warmup, 10)):
            sess.run_device()
        kernels.device_check(dev)
        n = 200
        ms_launch = time_loop(sess.run_device, n, world, stream) / n
        kernels.device_check(dev)
        # the same step replayed from a CUDA graph: one host call instead of two Python launches
        graph = sess.capture()
        for _ in range(3):
            graph.replay()
        ms = time_loop(graph.replay, n, world, stream) / n
        kernels.device_check(dev)
        ref = sess.run_device().clone()
        graph.replay()
        same = bool(torch.equal(ref, sess.o))
        fl = causal_flops(1, HQ, S, D)  # every rank runs its heads of the one sequence
        out[key] = {"seq_len": S, "batch": 1, "ms_per_step": ms, "value": fl / (ms * 1e-3) / 1e12,
                    "unit": "TFLOP/s", "steps": n, "launches_per_step": sess.launches_per_step(),
                    "launch": "CUDA graph replay (PrefillSession.capture)", "graph_equals_direct": same,
                    "ms_per_step_direct_launches": ms_launch,
                    "l2": "inputs fit in L2 (no flush between steps)"}
        del graph, sess
    return out


def run_reference(args, world, rank):
    if rank != 0:
        return 0
    samples = []
    for _ in range(max(args.warmup, 0)):
        cpu_reference_sample(1, S_PREFILL)
        break
    tot_t, tot_f = 0.0, 0.0
    for _ in range(args.steps):
        dt, fl, cores = cpu_reference_sample(1, S_PREFILL)
        tot_t += dt
        tot_f += fl
        samples.append(dt)
    val = tot_f / tot_t / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * tot_t / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": "gqa_causal_prefill", "sample": "1 query head (kv head 0) of batch element 0 per step",
                   "seq_len": S_PREFILL, "q_heads": HQ, "kv_heads": HKV, "head_dim": D},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": "one (batch, q-head) of the seq-8192 workload per step; NumPy fp32 per-head "
                                   "QK^T, triu mask, softmax, PV (CPU_Baseline gqa_attention_cpu restated)"},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, world, rank, local):
    from llama3_8b_attention_optimize_b200 import kernels
    from llama3_8b_attention_optimize_b200.session import DecodeSession, PrefillSession, PrefillStream
    from llama3_8b_attention_optimize_b200.shard import kv_shard

    sh = kv_shard(rank, world, HKV, HQ)
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)
    B = B_PER_GPU * world  # global batch; this rank owns sh.kv_count kv heads of every sequence
    hq, hkv = sh.q_count, sh.kv_count

    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    sess = PrefillSession(B, S_PREFILL, hq, hkv, D, causal=True, rope=args.rope, device=dev)
    sess.q.copy_(torch.randn(sess.shape_q, generator=gen, device=dev) * 2.5)
    sess.k.copy_(torch.randn(sess.shape_kv, generator=gen, device=dev) * 2.5)
    sess.v.copy_(torch.randn(sess.shape_kv, generator=gen, device=dev))

    for _ in range(args.warmup):
        sess.run_device()
    kernels.device_check(dev)
    flops_rank = causal_flops(B, hq, S_PREFILL, D)
    with ClockSampler(local) as clk:
        t_a = time.monotonic()
        ms = time_loop(sess.run_device, args.steps, world, stream)
        clk.window(t_a, time.monotonic())
    kernels.device_check(dev)
    ms_step = ms / args.steps
    flops_total = causal_flops(B, HQ, S_PREFILL, D)
    value = flops_total / (ms_step * 1e-3) / 1e12

    # ---- the same step back to back for >= 2 s: the clock the power cap settles at
    sustained = None
    if args.sustained_s > 0:
        n_sus = max(args.steps, int(args.sustained_s * 1e3 / ms_step) + 1)
        with ClockSampler(local) as clk_s:
            t_a = time.monotonic()
            ms_sus = time_loop(sess.run_device, n_sus, world, stream)
            clk_s.window(t_a, time.monotonic())
        kernels.device_check(dev)
        sustained = {"value": flops_total / (ms_sus / n_sus * 1e-3) / 1e12, "unit": "TFLOP/s",
                     "ms_per_step": ms_sus / n_sus, "steps": n_sus, "timed_s": ms_sus * 1e-3,
                     "clocks": clk_s.summary()}

    # ---- the smaller prefill configurations (one sequence, one GPU's share of heads):
    # S=128 (the reference's CPU-runnable core) and S=2048, same mode as the headline
    short = run_short_prefills(args, hq, hkv, dev, stream, world)

    # ---- end to end through the host-buffer API (pinned host in, pinned host out); every
    # step copies its Q/K/V in and its O out, overlapped across steps on three streams
    qh = sess.q.to("cpu").pin_memory()
    kh = sess.k.to("cpu").pin_memory()
    vh = sess.v.to("cpu").pin_memory()
    ohs = [torch.empty(sess.shape_q, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    e2e_steps = max(2, min(args.steps, 12))
    pipe = PrefillStream(B, S_PREFILL, hq, hkv, D, causal=True, rope=args.rope, device=dev)
    del sess
    pipe.run([(qh, kh, vh, ohs[i % 2]) for i in range(2)])
    torch.cuda.synchronize()
    ms_e2e = time_loop(lambda: pipe.run([(qh, kh, vh, ohs[i % 2]) for i in range(e2e_steps)]), 1, world,
                       stream) / e2e_steps
    e2e_value = flops_total / (ms_e2e * 1e-3) / 1e12
    e2e_h2d, e2e_d2h, e2e_launches = pipe.h2d_bytes(), pipe.d2h_bytes(), pipe.launches_per_step()
    del qh, kh, vh, ohs, pipe

    # ---- split-KV decode (HBM-bound), same sharding
    dB = DEC_B * world
    dgen = torch.Generator().manual_seed(99)
    lens_all = torch.randint(1024, DEC_LMAX + 1, (dB,), generator=dgen, dtype=torch.int32)
    ds = DecodeSession(dB, DEC_LMAX, hq, hkv, D, device=dev)
    kc = torch.empty(dB, hkv, DEC_LMAX, D, dtype=torch.bfloat16, device=dev)
    vc = torch.empty_like(kc)
    for b0 in range(0, dB, 8):
        kc[b0:b0 + 8].normal_(generator=gen)
        vc[b0:b0 + 8].normal_(generator=gen)
    ds.q.copy_(torch.randn(ds.q.shape, generator=gen, device=dev))
    ds.lens.copy_(lens_all.to(dev))
    for _ in range(args.warmup):
        ds.run_device(kc, vc)
    kernels.device_check(dev)
    dsteps = max(args.steps, 10)
    ms_dec = time_loop(lambda: ds.run_device(kc, vc), dsteps, world, stream) / dsteps
    kernels.device_check(dev)
    dec_bytes_rank = float(lens_all.sum().item()) * hkv * D * 2 * 2
    dec_bytes_total = float(lens_all.sum().item()) * HKV * D * 2 * 2
    dec_gbs = dec_bytes_total / (ms_dec * 1e-3) / 1e9
    paged = run_decode_paged(args, world, dev, stream, ds, kc, vc, lens_all, hkv, dec_bytes_total, ms_dec)
    del kc, vc

    # ---- full attention layer (S=4096, hidden 4096): q/k/v projection with RoPE in the
    # epilogue, causal core, o_proj (+ fp32 all-reduce across ranks): strong scaling
    layer = run_layer(args, world, rank, dev, stream)

    hbm_peak, tc_peak, tc_sust, peak_src = load_peaks()
    prof = load_profile_traffic()
    achieved = flops_rank / (ms_step * 1e-3) / 1e12
    roof = {"bound": "tensor", "achieved": achieved, "peak": tc_peak, "unit": "TFLOP/s",
            "frac": achieved / tc_peak, "peak_source": f"{peak_src} bf16 dense (burst)",
            "traffic": prof.get("prefill_bytes_per_launch"),
            "algorithmic_flops_per_launch": flops_rank}
    dec_ach = dec_bytes_rank / (ms_dec * 1e-3) / 1e9
    dec_roof = {"bound": "hbm", "achieved": dec_ach, "peak": hbm_peak, "unit": "GB/s", "frac": dec_ach / hbm_peak,
                "traffic": prof.get("decode_bytes_per_launch"), "algorithmic_bytes_per_launch": dec_bytes_rank}

    if rank != 0:
        return 0
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        dt, fl, cores = cpu_reference_sample(24, S_PREFILL)
        cpu = {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
               "sample": "24 query heads (kv head 0, batch element 0) of the seq-8192 workload, NumPy fp32 "
                         "(CPU_Baseline gqa_attention_cpu restated), %.1f s" % dt}
        cpu.update(cpu_small_configs())
        for key, gpu in (("c1", short["c1"]), ("c2", short["c2"])):
            cpu[f"{key}_gpu_ms"] = gpu["ms_per_step"]
            cpu[f"{key}_speedup"] = cpu[f"{key}_ms"] / gpu["ms_per_step"]
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1); Q,K x2.5)",
        "config": {"workload": "gqa_causal_prefill_from_unrotated_qk", "rope": args.rope,
                   "global_batch": B, "batch_per_gpu_equiv": B_PER_GPU,
                   "seq_len": S_PREFILL, "q_heads": HQ, "kv_heads": HKV, "head_dim": D,
                   "parallelism": f"kv_head_shard{world}", "l2": "inputs 335 MB/rank > L2 (126 MB)"},
        "roofline": roof,
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "ms_per_step": ms_e2e, "steps": e2e_steps,
                "h2d_bytes_per_step": e2e_h2d * world, "d2h_bytes_per_step": e2e_d2h * world,
                "path": "PrefillStream.run: per step pinned host Q/K/V -> device, K pre-pass + gqa_prefill_bf16, "
                        "O -> pinned host; copies of neighbouring steps overlap the compute"},
        "gpu_launches": args.steps * e2e_launches,
        "clocks": clk.summary(),
        "decode": {"metric": "split-KV GQA decode HBM GB/s", "value": dec_gbs, "unit": "GB/s", "ms_per_step": ms_dec,
                   "config": {"batch": dB, "max_len": DEC_LMAX, "lens": "U[1024,32768] seed 99",
                              "kv_heads_per_gpu": hkv}, "roofline": dec_roof, "gpu_launches": 2 * dsteps},
        "decode_paged": paged,
        "full_layer": layer,
        "short_prefill": short,
    }
    if sustained is not None:
        sustained["frac_of_sustained_peak"] = (sustained["value"] / world) / tc_sust if tc_sust else None
        sustained["frac_of_burst_peak"] = (sustained["value"] / world) / tc_peak
        line["sustained"] = sustained
    lt = layer["achieved_per_gpu"]
    layer["roofline"] = {"bound": "tensor", "achieved": lt, "peak": tc_peak, "unit": "TFLOP/s", "frac": lt / tc_peak}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


def run_decode_paged(args, world, dev, stream, ds, kc, vc, lens_all, hkv, dec_bytes_total, ms_dec) -> dict:
    """The decode workload over a paged cache: the same rows scattered into shuffled
    128-key pages (pool sized to the sequences, one spare row each), decoded through the
    block table; plus the per-step RoPE-on-append of one new token per sequence."""
    from llama3_8b_attention_optimize_b200 import kernels

    P = 128
    dB = kc.shape[0]
    n_lp = [(int(L) + 1 + P - 1) // P for L in lens_all.tolist()]
    max_pages = max(n_lp)
    perm = torch.randperm(sum(n_lp), generator=torch.Generator().manual_seed(7)).to(torch.int32)
    table_h = torch.full((dB, max_pages), -1, dtype=torch.int32)
    kp = torch.empty(sum(n_lp), hkv, P, D, dtype=torch.bfloat16, device=dev)
    vp = torch.empty_like(kp)
    off = 0
    for b in range(dB):
        n = n_lp[b]
        ids = perm[off:off + n]
        table_h[b, :n] = ids
        nc = min(n, kc.shape[2] // P)  # a full sequence's spare row lives in a page of its own
        idx = ids[:nc].to(dev, torch.long)
        kp[idx] = kc[b, :, :nc * P].reshape(hkv, nc, P, D).transpose(0, 1)
        vp[idx] = vc[b, :, :nc * P].reshape(hkv, nc, P, D).transpose(0, 1)
        off += n
    table = table_h.to(dev)
    ws = torch.empty(max(kernels.decode_workspace_bytes(dB, ds.Hq, max_pages * P), 16), dtype=torch.uint8,
                     device=dev)
    cos, sin = kernels.rope_cache(max_pages * P + 1, device=dev)

    def step():
        kernels.decode_paged(ds.q, kp, vp, table, ds.lens, q_pos=ds.lens, cos=cos, sin=sin, workspace=ws,
                             out=ds.o)

    for _ in range(args.warmup):
        step()
    ref = ds.run_device(kc, vc).clone()
    step()
    kernels.device_check(dev)
    identical = bool(torch.equal(ds.o, ref))
    dsteps = max(args.steps, 10)
    ms = time_loop(step, dsteps, world, stream) / dsteps
    # one new token per sequence per step: K rotated at lens[b] and written into its page
    kn = torch.randn(dB, hkv, 1, D, device=dev).to(torch.bfloat16)
    vn = torch.randn(dB, hkv, 1, D, device=dev).to(torch.bfloat16)

    def app():
        kernels.kv_append(kn, vn, kp, vp, ds.lens, cos=cos, sin=sin, block_table=table)

    for _ in range(args.warmup):
        app()
    ms_app = time_loop(app, dsteps, world, stream) / dsteps
    kernels.device_check(dev)
    del kp, vp
    return {"metric": "paged split-KV GQA decode HBM GB/s", "value": dec_bytes_total / (ms * 1e-3) / 1e9,
            "unit": "GB/s", "ms_per_step": ms, "vs_contiguous": ms_dec / ms, "bit_identical_to_contiguous": identical,
            "config": {"page_size": P, "pages": int(sum(n_lp)), "layout": "[pages][kv_heads][128 keys][128]",
                       "assignment": "shuffled (seed 7)"},
            "append_us_per_step": ms_app * 1e3,
            "append_config": "1 token x %d sequences x %d kv heads, RoPE at lens[b], paged" % (dB, hkv),
            "gpu_launches": 2 * dsteps + dsteps}


# Largest rank counts the NVLink peer-memory o_proj exchanges have been run and checked
# on (tests/test_gpu_tp_peer.py at 2, 4 and 8 ranks against the NCCL path and the
# float64 sum of the partials; this bench reports each variant's difference from NCCL).
P2P_FUSED_CHECKED_RANKS = 8
P2P_CHECKED_RANKS = 8


def run_layer(args, world, rank, dev, stream) -> dict:
    from llama3_8b_attention_optimize_b200 import kernels
    from llama3_8b_attention_optimize_b200.layer import FullLayerSession, reduce_partials

    ls = FullLayerSession(LAYER_S, rank=rank, world=world, device=dev)
    g = torch.Generator(device=dev).manual_seed(4242)  # identical weights and input on every rank
    wq = (torch.randn(4096, 4096, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wk = (torch.randn(1024, 4096, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wv = (torch.randn(1024, 4096, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wo = (torch.randn(4096, 4096, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    ls.set_weights(wq, wk, wv, wo)
    ls.h.copy_(torch.randn(ls.h.shape, generator=g, device=dev))
    del wq, wk, wv, wo
    for _ in range(args.warmup):
        ls.run_device()
    kernels.device_check(dev)
    lsteps = max(args.steps // 4, 10)
    ms = time_loop(ls.run_device, lsteps, world, stream) / lsteps
    kernels.device_check(dev)
    fl = ls.flops()
    out = {"metric": "attention layer TFLOP/s (q/k/v proj + RoPE + causal GQA core + o_proj)", "unit": "TFLOP/s",
           "value": fl["total"] / (ms * 1e-3) / 1e12, "ms_per_step": ms, "steps": lsteps, "scaling": "strong",
           "achieved_per_gpu": fl["total"] / world / (ms * 1e-3) / 1e12,
           "config": {"seq_len": LAYER_S, "batch": 1, "hidden": 4096, "q_heads": HQ, "kv_heads": HKV,
                      "parallelism": f"kv_head_shard{world} (column-parallel qkv, row-parallel o_proj)",
                      "flops": fl},
           "gpu_launches": lsteps * (3 if world == 1 else 4)}
    if world > 1:
        ar = time_loop(lambda: reduce_partials(ls.partial, world), lsteps, world, stream) / lsteps
        nbytes = ls.partial.numel() * 4
        out["all_reduce"] = {"ms": ar, "bytes": nbytes, "dtype": "fp32",
                             "bus_gbs": nbytes * 2 * (world - 1) / world / (ar * 1e-3) / 1e9}
        # other ways to combine the row-parallel partials, each checked against the step above:
        # reduce-scatter fp32 + round + all-gather bf16; o_proj and all-reduce pipelined
        # over row chunks (GEMM grid capped so NCCL finds free SMs)
        ls.run_device()
        ref = ls.out.clone()
        variants = []
        # peer-memory exchanges run only at rank counts they have been checked on
        checked_up_to = {"p2p_fused": P2P_FUSED_CHECKED_RANKS, "p2p": P2P_CHECKED_RANKS}
        for mode, chunks, ctas in (("p2p_fused", 1, 0), ("p2p", 1, 0), ("rs_ag", 1, 0), ("all_reduce", 4, 132)):
            if world > checked_up_to.get(mode, world):
                variants.append({"reduce": mode, "skipped": f"checked on up to {checked_up_to[mode]} GPUs"})
                continue
            try:  # raised on every rank together when peer mapping is unavailable
                lc = FullLayerSession(LAYER_S, rank=rank, world=world, device=dev, o_chunks=chunks, gemm_ctas=ctas,
                                      reduce=mode)
            except RuntimeError as exc:
                variants.append({"reduce": mode, "unavailable": str(exc)[:200]})
                continue
            for dst, src in ((lc.wq, ls.wq), (lc.wk, ls.wk), (lc.wv, ls.wv), (lc.wo, ls.wo), (lc.h, ls.h)):
                dst.copy_(src)
            for _ in range(args.warmup):
                lc.run_device()
            kernels.device_check(dev)
            diff = float((lc.out.float() - ref.float()).abs().max().item())
            msc = time_loop(lc.run_device, lsteps, world, stream) / lsteps
            kernels.device_check(dev)
            variants.append({"reduce": mode, "chunks": len(lc.chunks), "gemm_ctas": ctas or "all",
                             "ms_per_step": msc, "value": fl["total"] / (msc * 1e-3) / 1e12,
                             "max_abs_diff_vs_all_reduce": diff})
            if mode == "p2p":  # the exchange alone, on a partial already in the buffer
                lc.peer.reduce_gather()
                variants[-1]["exchange_ms"] = time_loop(lc.peer.reduce_gather, lsteps, world, stream) / lsteps
                kernels.device_check(dev)
            lc.close()
            del lc
        out["variants"] = variants
        timed = [v for v in variants if "ms_per_step" in v]
        if timed:  # the fastest way to combine the partials, next to the NCCL step above
            best = min(timed, key=lambda v: v["ms_per_step"])
            if best["ms_per_step"] < ms:
                out["best"] = {"reduce": best["reduce"], "ms_per_step": best["ms_per_step"], "value": best["value"]}
    del ls
    return out


def run_profile_case(args):
    """Small cases for ncu captures (inputs > L2, a few hundred MB on the device):
    prefill: B=2, seq 8192, 32/8 heads, fused RoPE; decode: B=8, cache 32768 keys;
    decode_paged: the same decode over shuffled 128-key pages, plus one RoPE-on-append of a
    token per sequence; gemm: the projection GEMM at 4096 x 4096 x 4096 (bf16 out)."""
    from llama3_8b_attention_optimize_b200 import kernels
    from llama3_8b_attention_optimize_b200.session import DecodeSession, PrefillSession
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(7)
    if args.profile_case == "gemm":
        x = (torch.randn(4096, 4096, generator=gen, device=dev)).to(torch.bfloat16)
        w = (torch.randn(4096, 4096, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        y = torch.empty(4096, 4096, dtype=torch.bfloat16, device=dev)
        fn = lambda: kernels.linear(x, w, out=y)  # noqa: E731
    elif args.profile_case == "prefill":
        sess = PrefillSession(2, S_PREFILL, HQ, HKV, D, rope=args.rope, device=dev)
        sess.q.copy_(torch.randn(sess.shape_q, generator=gen, device=dev) * 2.5)
        sess.k.copy_(torch.randn(sess.shape_kv, generator=gen, device=dev) * 2.5)
        sess.v.copy_(torch.randn(sess.shape_kv, generator=gen, device=dev))
        fn = sess.run_device
    else:
        B = 8
        ds = DecodeSession(B, DEC_LMAX, HQ, HKV, D, device=dev)
        kc = torch.randn(B, HKV, DEC_LMAX, D, generator=gen, device=dev).to(torch.bfloat16)
        vc = torch.randn(B, HKV, DEC_LMAX, D, generator=gen, device=dev).to(torch.bfloat16)
        ds.q.copy_(torch.randn(ds.q.shape, generator=gen, device=dev))
        lens = torch.randint(1024, DEC_LMAX + 1, (B,), generator=torch.Generator().manual_seed(99), dtype=torch.int32)
        ds.lens.copy_(lens.to(dev))
        fn = lambda: ds.run_device(kc, vc)  # noqa: E731
        if args.profile_case == "decode_paged":
            P, n_lp = 128, DEC_LMAX // 128
            perm = torch.randperm(B * n_lp, generator=torch.Generator().manual_seed(7)).to(torch.int32)
            table = perm.view(B, n_lp).to(dev)
            kp = kc.view(B, HKV, n_lp, P, D).transpose(1, 2).reshape(B * n_lp, HKV, P, D)
            vp = vc.view(B, HKV, n_lp, P, D).transpose(1, 2).reshape(B * n_lp, HKV, P, D)
            kpool, vpool = torch.empty_like(kp), torch.empty_like(vp)
            kpool[perm.to(dev, torch.long)] = kp
            vpool[perm.to(dev, torch.long)] = vp
            del kp, vp, kc, vc
            kn = torch.randn(B, HKV, 1, D, generator=gen, device=dev).to(torch.bfloat16)
            short = (ds.lens - 1).clamp(min=0)  # append into the last cached row: stays in the pool

            def fn():
                kernels.kv_append(kn, kn, kpool, vpool, short, cos=ds.cos, sin=ds.sin, block_table=table)
                kernels.decode_paged(ds.q, kpool, vpool, table, ds.lens, q_pos=ds.lens, cos=ds.cos, sin=ds.sin,
                                     workspace=ds.ws, out=ds.o)
    for _ in range(args.warmup + args.steps):
        fn()
    kernels.device_check(dev)
    print(f"profile case {args.profile_case}: {args.warmup + args.steps} launches ok")
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--profile-case", choices=["prefill", "decode", "decode_paged", "gemm"], default=None,
                    help="run a small case for ncu captures instead of the benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sustained-s", type=float, default=2.0,
                    help="also time the headline step back to back for this many seconds (0: skip)")
    ap.add_argument("--rope", choices=["prepass_k", "fused", "none"], default="prepass_k",
                    help="prepass_k: K rotated once by its own kernel, Q rotated inside the fused kernel; "
                         "fused: both rotated inside the fused kernel")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.profile_case:
        return run_profile_case(args)
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        return run_reference(args, world, rank)
    world, rank, local = dist_setup(args)
    try:
        return run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
