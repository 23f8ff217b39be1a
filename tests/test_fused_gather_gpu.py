"""Fused GEMM + all-gather through peer memory (bw_gemm_*_allgather): every rank's C_full must
equal the shards that the plain single-GPU GEMM computes, gathered by NCCL and unsharded
(bit-identical: same kernel, same tiles), plus a direct oracle check of this rank's columns.
One process per GPU over all visible GPUs (up to 4); world = 1 runs on any box."""
import os
import socket

import numpy as np
import pytest

import bwgemm
import oracle as o

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, kind):
    import torch
    import torch.distributed as dist

    import sharding

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        bwgemm.init(rank)
        M, K, ns = 512, 1024, 256
        N = ns * world
        if kind == "f16":
            A = torch.from_numpy(o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((M, K), 301)))).to(dev).half()
            Bf = o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((K, N), 302)))
            Bs = torch.from_numpy(np.ascontiguousarray(Bf[:, rank * ns:(rank + 1) * ns])).to(dev).half()
            sym = sharding.SymmetricC(M, N, torch.float32, dev, world, rank)
            dist.barrier()
            bwgemm.gemm_f16_allgather(A, Bs, sym.C, sym.peers, rank)
            mine = bwgemm.gemm_f16(A, Bs)
        else:
            Af = o.seeded_normal((M, K), 303)
            Bf = o.seeded_normal((K, N), 304)
            qa, sa = bwgemm.quantize_fp8(torch.from_numpy(Af).to(dev), False, bwgemm.SCALE_AMAX)
            qb, sb = bwgemm.quantize_fp8(torch.from_numpy(Bf).to(dev), True, bwgemm.SCALE_AMAX)  # N x K
            qbs = qb[rank * ns:(rank + 1) * ns].contiguous()
            sym = sharding.SymmetricC(M, N, torch.bfloat16, dev, world, rank)
            dist.barrier()
            bwgemm.gemm_fp8_allgather(qa, qbs, sa, sb, sym.C, sym.peers, rank, bwgemm.OUT_BF16)
            mine = bwgemm.gemm_fp8(qa, qbs, sa, sb, out_dtype=bwgemm.OUT_BF16)
        torch.cuda.synchronize()
        assert bwgemm.device_status() == 0
        dist.barrier()  # every rank's stores into every C_full have completed
        gathered = sharding.gather_columns(mine, world)
        torch.cuda.synchronize()
        assert torch.equal(sym.C, gathered), f"rank {rank}: fused gather differs from NCCL gather"
        if kind == "f16":
            R = o.gemm_f64(o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((M, K), 301))), Bf)
            tol = o.f16_tolerance(K, 1.0, 1.0)
            assert np.abs(sym.C.cpu().numpy() - R).max() <= tol
        dist.barrier()
        sym.close()
    finally:
        dist.destroy_process_group()


def _ngpus():
    import torch

    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return [1] + ([min(4, n)] if n >= 2 else [])


@pytest.mark.parametrize("world", _ngpus())
@pytest.mark.parametrize("kind", ["f16", "fp8"])
def test_fused_allgather(cuda_dev, world, kind):
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(world, _free_port(), kind), nprocs=world, start_method="spawn", join=True)


def test_fused_allgather_rejects_misaligned_shards(cuda_dev):
    import torch

    A = torch.zeros((64, 64), dtype=torch.float16, device=cuda_dev)
    B = torch.zeros((64, 12), dtype=torch.float16, device=cuda_dev)  # 12 FP32 columns: 48-byte rows
    C = torch.zeros((64, 24), dtype=torch.float32, device=cuda_dev)
    with pytest.raises(bwgemm.BwError):
        bwgemm.gemm_f16_allgather(A, B, C, [None, 0], 0)


@pytest.mark.parametrize("kind", ["f16", "fp8_f32", "fp8_bf16"])
@pytest.mark.parametrize("M,ns,K", [(300, 136, 208), (512, 256, 1024), (1024, 520, 512)])
def test_multicast_epilogue_indexing_with_plain_stores(cuda_dev, monkeypatch, kind, M, ns, K):
    """The multicast gather's epilogue (16-byte pieces of the staged chunks, clipped to C) with
    BW_MC_PLAIN=1, i.e. plain stores into an ordinary buffer, on one GPU: the calls of all
    `world` ranks together must fill C_full with exactly the shards the plain GEMM computes.
    This is the single-GPU check of the indexing the multimem stores use."""
    import torch

    monkeypatch.setenv("BW_MC_PLAIN", "1")
    world = 4
    N = ns * world
    if kind == "f16":
        A = torch.from_numpy(o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((M, K), 311)))).to(cuda_dev).half()
        B = torch.from_numpy(o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((K, N), 312)))).to(cuda_dev).half()
        C = torch.full((M, N), float("nan"), device=cuda_dev)
        for r in range(world):
            Bs = B[:, r * ns:(r + 1) * ns].contiguous()
            bwgemm.gemm_f16_allgather_multicast(A, Bs, C.data_ptr(), world, r, N)
        want = torch.cat([bwgemm.gemm_f16(A, B[:, r * ns:(r + 1) * ns].contiguous()) for r in range(world)], dim=1)
    else:
        out = bwgemm.OUT_F32 if kind == "fp8_f32" else bwgemm.OUT_BF16
        dt = torch.float32 if out == bwgemm.OUT_F32 else torch.bfloat16
        qa, sa = bwgemm.quantize_fp8(torch.from_numpy(o.seeded_normal((M, K), 313)).to(cuda_dev), False)
        qb, sb = bwgemm.quantize_fp8(torch.from_numpy(o.seeded_normal((K, N), 314)).to(cuda_dev), True)
        C = torch.full((M, N), float("nan"), device=cuda_dev, dtype=dt)
        for r in range(world):
            bwgemm.gemm_fp8_allgather_multicast(qa, qb[r * ns:(r + 1) * ns].contiguous(), sa, sb, C.data_ptr(), world,
                                                r, N, out)
        want = torch.cat([bwgemm.gemm_fp8(qa, qb[r * ns:(r + 1) * ns].contiguous(), sa, sb, out_dtype=out)
                          for r in range(world)], dim=1)
    torch.cuda.synchronize()
    assert bwgemm.device_status() == 0
    assert torch.equal(C, want)


def _mc_worker(rank, world, port, kind):
    import torch
    import torch.distributed as dist

    import sharding

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        bwgemm.init(rank)
        M, K, ns = 640, 1024, 264
        N = ns * world
        dt = torch.float32 if kind == "f16" else torch.bfloat16
        mcC = sharding.MulticastC(M, N, dt, dev)
        if not mcC.available:
            return
        mcC.C.fill_(float("nan"))
        torch.cuda.synchronize()
        dist.barrier()
        if kind == "f16":
            A = torch.from_numpy(o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((M, K), 321)))).to(dev).half()
            Bf = o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((K, N), 322)))
            Bs = torch.from_numpy(np.ascontiguousarray(Bf[:, rank * ns:(rank + 1) * ns])).to(dev).half()
            bwgemm.gemm_f16_allgather_multicast(A, Bs, mcC.mc, world, rank, N)
            mine = bwgemm.gemm_f16(A, Bs)
        else:
            qa, sa = bwgemm.quantize_fp8(torch.from_numpy(o.seeded_normal((M, K), 323)).to(dev), False)
            qb, sb = bwgemm.quantize_fp8(torch.from_numpy(o.seeded_normal((K, N), 324)).to(dev), True)
            qbs = qb[rank * ns:(rank + 1) * ns].contiguous()
            bwgemm.gemm_fp8_allgather_multicast(qa, qbs, sa, sb, mcC.mc, world, rank, N, bwgemm.OUT_BF16)
            mine = bwgemm.gemm_fp8(qa, qbs, sa, sb, out_dtype=bwgemm.OUT_BF16)
        torch.cuda.synchronize()
        assert bwgemm.device_status() == 0
        dist.barrier()
        gathered = sharding.gather_columns(mine, world)
        torch.cuda.synchronize()
        ok = bool(torch.equal(mcC.C, gathered))
        flag = torch.tensor([0.0 if ok else 1.0], device=dev)
        dist.all_reduce(flag)
        torch.cuda.synchronize()
        dist.barrier()
        # every rank reaches this point before any rank can fail, so no rank leaves while the
        # others still hold the multicast binding
        assert float(flag.item()) == 0.0, f"rank {rank}: multicast gather differs from NCCL gather"
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["f16", "fp8"])
def test_multicast_allgather(cuda_dev, kind):
    """Fused GEMM + all-gather with multimem stores on all visible GPUs (up to 4; needs 2)."""
    import torch
    import torch.multiprocessing as mp

    n = min(4, torch.cuda.device_count())
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    mp.start_processes(_mc_worker, args=(n, _free_port(), kind), nprocs=n, start_method="spawn", join=True)


@pytest.mark.parametrize("staging", ["2", "6"])
@pytest.mark.parametrize("kind", ["f16", "fp8"])
def test_fused_allgather_emulated_ranks_on_one_gpu(cuda_dev, monkeypatch, staging, kind):
    """The peer-store gather with `world` ranks emulated on one GPU: each rank's C_full is an
    ordinary local buffer and every rank's call gets the others' buffers as its peers, so the
    calls one after another fill every C_full. Covers both staging depths of the epilogue
    (BW_GATHER_STAGING: 2 buffers a warp with 3 pipeline stages, or 6 with 2)."""
    import torch

    monkeypatch.setenv("BW_GATHER_STAGING", staging)
    world, M, K, ns = 3, 520, 640, 264
    N = ns * world
    if kind == "f16":
        A = torch.from_numpy(o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((M, K), 331)))).to(cuda_dev).half()
        B = torch.from_numpy(o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((K, N), 332)))).to(cuda_dev).half()
        Cs = [torch.full((M, N), float("nan"), device=cuda_dev) for _ in range(world)]
        for r in range(world):
            peers = [None if q == r else Cs[q].data_ptr() for q in range(world)]
            bwgemm.gemm_f16_allgather(A, B[:, r * ns:(r + 1) * ns].contiguous(), Cs[r], peers, r)
        want = bwgemm.gemm_f16(A, B)
    else:
        qa, sa = bwgemm.quantize_fp8(torch.from_numpy(o.seeded_normal((M, K), 333)).to(cuda_dev), False)
        qb, sb = bwgemm.quantize_fp8(torch.from_numpy(o.seeded_normal((K, N), 334)).to(cuda_dev), True)
        Cs = [torch.full((M, N), float("nan"), device=cuda_dev, dtype=torch.bfloat16) for _ in range(world)]
        for r in range(world):
            peers = [None if q == r else Cs[q].data_ptr() for q in range(world)]
            bwgemm.gemm_fp8_allgather(qa, qb[r * ns:(r + 1) * ns].contiguous(), sa, sb, Cs[r], peers, r,
                                      bwgemm.OUT_BF16)
        want = torch.cat([bwgemm.gemm_fp8(qa, qb[r * ns:(r + 1) * ns].contiguous(), sa, sb, out_dtype=bwgemm.OUT_BF16)
                          for r in range(world)], dim=1)
    torch.cuda.synchronize()
    assert bwgemm.device_status() == 0
    for C in Cs:
        assert torch.equal(C, want)
