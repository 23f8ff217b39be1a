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
