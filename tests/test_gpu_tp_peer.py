"""The tensor-parallel o_proj reduction over NVLink peer memory.

* gqa_tp_reduce_gather_bf16 (pull) and gqa_tp_o_proj_exchange_bf16 (fused push) give the
  same layer output, step after step, at 2, 4 and 8 ranks (each size skipped when the box
  has fewer GPUs): bit-identical to the NCCL all-reduce path at 2 ranks (an fp32 sum of
  two terms does not depend on the order), and at every size within one bf16 ulp of the
  float64 sum of all ranks' partials plus the fp32 summation error (world - 1 additions
  at 2^-24 of the partials' magnitudes: where the partials cancel, an fp32 sum is more
  than one bf16 ulp from the exact value, for NCCL's order too); NCCL is held to the same
  bound, and the ulp histogram of the exchange against the exact sum is printed.
* A peer that never signals -- a missing buffer on one GPU, or a rank that skips a step --
  ends the waits with GQA_ERR_DEVICE_TIMEOUT instead of a hang, on the pull and the fused
  path, and the GPU stays usable.
"""
import ctypes
import json
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llama3_8b_attention_optimize_b200 import _lib, kernels

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int):
    import sys
    sys.path.insert(0, ROOT)
    from datetime import timedelta

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    return dev


def _weights(dev):
    g = torch.Generator(device=dev).manual_seed(9)
    w = [(torch.randn(o, 4096, generator=g, device=dev) * 0.02).to(torch.bfloat16) for o in (4096, 1024, 1024, 4096)]
    return g, w


def _ulp_key(t: torch.Tensor) -> torch.Tensor:
    w = t.contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
    return torch.where(w >= 0x8000, 0x8000 - (w - 0x8000), 0x8000 + w)


def _worker(rank: int, world: int, port: int, out_dir: str):
    dev = _init(rank, world, port)
    from llama3_8b_attention_optimize_b200 import kernels as K
    from llama3_8b_attention_optimize_b200.layer import FullLayerSession

    try:
        S = 1024  # the fused exchange needs S / world to be a multiple of 128 rows
        g, (wq, wk, wv, wo) = _weights(dev)
        ref = FullLayerSession(S, rank=rank, world=world, device=dev)
        p2p = FullLayerSession(S, rank=rank, world=world, device=dev, reduce="p2p")
        fused = FullLayerSession(S, rank=rank, world=world, device=dev, reduce="p2p_fused")
        for sess in (ref, p2p, fused):
            sess.set_weights(wq, wk, wv, wo)
        hist = {"0": 0, "1": 0, ">1": 0}
        nccl_hist = {"0": 0, "1": 0, ">1": 0}
        for step in range(4):  # new input every step: no stale blocks survive an epoch
            h = torch.randn(ref.h.shape, generator=g, device=dev).to(torch.bfloat16)
            for sess in (ref, p2p, fused):
                sess.h.copy_(h)
            part = ref.run_partial().clone()
            a = ref.run_device().clone()
            b = p2p.run_device().clone()
            c = fused.run_device().clone()
            K.device_check(dev)
            # the correctly rounded sum of every rank's partial
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            stack = torch.stack(parts).double()
            exact64 = stack.sum(0)
            exact = exact64.float().to(torch.bfloat16)
            # one bf16 rounding of an fp32 sum: within one bf16 ulp of the exact sum plus the
            # fp32 summation error (world - 1 additions, 2^-24 of the running magnitudes each)
            ulp = torch.exp2(torch.floor(torch.log2(exact64.abs().clamp_min(2.0 ** -126))) - 7)
            allow = ulp + (world - 1) * 2.0 ** -24 * stack.abs().sum(0)
            assert torch.equal(b, c), (rank, step, (b.float() - c.float()).abs().max().item())
            for got, hh in ((c, hist), (a, nccl_hist)):
                d = (_ulp_key(got) - _ulp_key(exact)).abs()
                hh["0"] += int((d == 0).sum())
                hh["1"] += int((d == 1).sum())
                hh[">1"] += int((d > 1).sum())
                err = (got.double() - exact64).abs()
                assert bool((err <= allow).all()), (rank, step, float((err - allow).max()))
            if world == 2:
                assert torch.equal(a, b), (rank, step, (a.float() - b.float()).abs().max().item())
        # more than one ulp only where the partials cancel: a small share of the outputs
        assert hist[">1"] <= 1e-4 * sum(hist.values()), hist
        p2p.close()
        fused.close()
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump({"peer_vs_exact": hist, "nccl_vs_exact": nccl_hist}, f)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.timeout(900)
def test_peer_reduction_equals_all_reduce(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    hists = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    total = {k: sum(h["peer_vs_exact"][k] for h in hists) for k in ("0", "1", ">1")}
    n = sum(total.values())
    print(f"world {world}: peer exchange vs float64 sum: 0 ulp {total['0'] / n:.6f}, 1 ulp {total['1'] / n:.6f}, "
          f"more {total['>1'] / n:.2e}")


def _skip_worker(rank: int, world: int, port: int, out_dir: str):
    """Step 1 runs on both ranks; in step 2 rank 1 does not take part (it leaves the step
    between launches).  Rank 0's fused exchange must end with a reported timeout."""
    dev = _init(rank, world, port)
    from llama3_8b_attention_optimize_b200 import _lib as L
    from llama3_8b_attention_optimize_b200 import kernels as K
    from llama3_8b_attention_optimize_b200.layer import FullLayerSession

    try:
        S = 256
        g, (wq, wk, wv, wo) = _weights(dev)
        fused = FullLayerSession(S, rank=rank, world=world, device=dev, reduce="p2p_fused")
        fused.set_weights(wq, wk, wv, wo)
        fused.h.copy_(torch.randn(fused.h.shape, generator=g, device=dev).to(torch.bfloat16))
        fused.run_device()
        K.device_check(dev)
        dist.barrier()
        code = 0
        if rank == 0:
            fused.run_device()
            try:
                K.device_check(dev)
            except L.GqaError as e:
                code = e.code
            x = torch.ones(4, device=dev)
            assert float(x.sum()) == 4.0  # the context still works
        torch.cuda.synchronize(dev)
        dist.barrier()
        fused.close()
        with open(os.path.join(out_dir, f"rank{rank}.code"), "w") as f:
            f.write(str(code))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_rank_that_skips_a_step_makes_its_peer_report_a_timeout(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_skip_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    assert int((tmp_path / "rank0.code").read_text()) == _lib.GQA_ERR_DEVICE_TIMEOUT
    assert int((tmp_path / "rank1.code").read_text()) == 0


def test_missing_peer_times_out_with_an_error():
    """Rank 0 of a two-rank exchange whose 'peer' buffer never signals: the bounded wait
    gives up (about 2 s) and gqa_device_check reports it; the GPU stays usable."""
    lib = _lib.load()
    S, N = 256, 512
    nbytes = lib.gqa_tp_buffer_bytes(S, N)
    hb = lib.gqa_peer_handle_bytes()
    ptrs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        assert lib.gqa_peer_alloc(nbytes, ctypes.byref(p), ctypes.create_string_buffer(hb)) == 0
        ptrs.append(p.value)
    try:
        bases = (ctypes.c_void_p * 2)(*ptrs)
        rc = lib.gqa_tp_reduce_gather_bf16(bases, 2, 0, S, N, 1, kernels._stream(torch.device("cuda")))
        assert rc == 0
        with pytest.raises(_lib.GqaError) as ei:
            kernels.device_check()
        assert ei.value.code == _lib.GQA_ERR_DEVICE_TIMEOUT
        x = torch.ones(4, device="cuda")
        assert float(x.sum()) == 4.0  # the context still works
    finally:
        for p in ptrs:
            lib.gqa_peer_free(p)


def test_fused_exchange_with_missing_peer_times_out_with_an_error():
    """The fused o_proj exchange as rank 0 of two, both buffers on this GPU: the GEMM
    stores into both and raises rank 0's flags, but rank 1's flag never comes, so the
    owner's bounded wait gives up and gqa_device_check reports it; the GPU stays usable."""
    lib = _lib.load()
    S, N, Hq = 256, 512, 16
    nbytes = lib.gqa_tp_buffer_bytes(S, N)
    hb = lib.gqa_peer_handle_bytes()
    ptrs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        assert lib.gqa_peer_alloc(nbytes, ctypes.byref(p), ctypes.create_string_buffer(hb)) == 0
        ptrs.append(p.value)
    try:
        attn = torch.zeros(Hq, S, 128, dtype=torch.bfloat16, device="cuda")
        wo = torch.zeros(N, Hq * 128, dtype=torch.bfloat16, device="cuda")
        bases = (ctypes.c_void_p * 2)(*ptrs)
        rc = lib.gqa_tp_o_proj_exchange_bf16(attn.data_ptr(), wo.data_ptr(), Hq * 128, bases, 2, 0, S, Hq, 128, N, 1,
                                             kernels._stream(torch.device("cuda")))
        assert rc == 0, _lib.strerror(rc)
        with pytest.raises(_lib.GqaError) as ei:
            kernels.device_check()
        assert ei.value.code == _lib.GQA_ERR_DEVICE_TIMEOUT
        x = torch.ones(4, device="cuda")
        assert float(x.sum()) == 4.0
    finally:
        torch.cuda.synchronize()
        for p in ptrs:
            lib.gqa_peer_free(p)
