"""The tensor-parallel o_proj reduction over NVLink peer memory (gqa_tp_reduce_gather_bf16):
two ranks give the same layer output as the NCCL all-reduce path, step after step; and a
peer that never signals ends the wait with a reported error instead of a hang."""
import ctypes
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


def _worker(rank: int, world: int, port: int, out_dir: str):
    import sys
    sys.path.insert(0, ROOT)
    from datetime import timedelta

    from llama3_8b_attention_optimize_b200 import kernels as K
    from llama3_8b_attention_optimize_b200.layer import FullLayerSession

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        S = 512
        g = torch.Generator(device=dev).manual_seed(9)
        wq = (torch.randn(4096, 4096, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wk = (torch.randn(1024, 4096, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wv = (torch.randn(1024, 4096, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wo = (torch.randn(4096, 4096, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        ref = FullLayerSession(S, rank=rank, world=world, device=dev)
        p2p = FullLayerSession(S, rank=rank, world=world, device=dev, reduce="p2p")
        fused = FullLayerSession(S, rank=rank, world=world, device=dev, reduce="p2p_fused")
        for sess in (ref, p2p, fused):
            sess.set_weights(wq, wk, wv, wo)
        for step in range(4):  # new input every step: no stale blocks survive an epoch
            h = torch.randn(ref.h.shape, generator=g, device=dev).to(torch.bfloat16)
            for sess in (ref, p2p, fused):
                sess.h.copy_(h)
            a = ref.run_device().clone()
            b = p2p.run_device().clone()
            c = fused.run_device().clone()
            K.device_check(dev)
            assert torch.equal(a, b), (rank, step, (a.float() - b.float()).abs().max().item())
            assert torch.equal(a, c), (rank, step, (a.float() - c.float()).abs().max().item())
        p2p.close()
        fused.close()
        with open(os.path.join(out_dir, f"rank{rank}.ok"), "w") as f:
            f.write("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.timeout(600)
def test_two_rank_peer_reduction_equals_all_reduce(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    assert all((tmp_path / f"rank{r}.ok").exists() for r in range(world))


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
