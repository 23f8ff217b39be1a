"""Column sharding of C = A x B over the GPUs of one node (one process per GPU).

Rank r owns columns [r * N/world, (r+1) * N/world) of B and C and runs the single-GPU GEMM on
them: no communication inside the GEMM. A gathered C, when requested, is an all-gather of the
M x (N/world) shards, which torch.distributed / NCCL deliver shard-major ([world][M][N/world]);
`unshard` permutes that into row-major M x N (on CUDA through bw_unshard_columns, elsewhere with
a tensor permute). The reference runs on one GPU only; this layer is new.
"""
from __future__ import annotations


def shard_bounds(N: int, world: int, rank: int) -> tuple[int, int]:
    """Column range of `rank`; N must divide evenly (the kernels need N % 8 == 0 per shard)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    if N % world:
        raise ValueError(f"N={N} is not divisible by world={world}")
    ns = N // world
    return rank * ns, (rank + 1) * ns


def local_shard(B, world: int, rank: int):
    """This rank's contiguous copy of B[:, shard]."""
    lo, hi = shard_bounds(B.shape[1], world, rank)
    return B[:, lo:hi].contiguous()


def unshard(C_shardmajor, M: int, N: int, world: int, out=None):
    """[world][M][N/world] -> row-major M x N."""
    if C_shardmajor.is_cuda:
        import bwgemm

        return bwgemm.unshard_columns(C_shardmajor.contiguous(), M, N, world, out=out)
    full = C_shardmajor.reshape(world, M, N // world).permute(1, 0, 2).reshape(M, N)
    if out is not None:
        out.copy_(full)
        return out
    return full.contiguous()


def gather_columns(C_local, world: int, group=None):
    """All-gather every rank's M x (N/world) shard and return the row-major M x N result."""
    import torch
    import torch.distributed as dist

    M, ns = C_local.shape
    if world == 1:
        return C_local
    buf = torch.empty((world * M, ns), dtype=C_local.dtype, device=C_local.device)
    dist.all_gather_into_tensor(buf, C_local.contiguous(), group=group)
    return unshard(buf, M, ns * world, world)


class SymmetricC:
    """Row-major M x N_total C that every rank holds in an IPC-shareable buffer, plus the peers'
    buffers mapped into this process: the target of the fused GEMM + all-gather
    (bwgemm.gemm_*_allgather). Handles are exchanged with torch.distributed.all_gather_object."""

    def __init__(self, M: int, N_total: int, dtype, device, world: int, rank: int, group=None):
        import torch.distributed as dist

        import bwgemm

        self.buf = bwgemm.IpcBuffer((M, N_total), dtype, device)
        self.C = self.buf.tensor
        self.rank, self.world = rank, world
        handles = [None] * world
        if world > 1:
            dist.all_gather_object(handles, self.buf.handle, group=group)
        self.peers = [None if q == rank else bwgemm.ipc_open(handles[q], device) for q in range(world)]

    def close(self):
        import bwgemm

        for p in self.peers:
            if p:
                bwgemm.ipc_close(p)
        self.peers = []
        self.buf.close()


class MulticastC:
    """Row-major M x N_total C in torch symmetric memory, bound on every rank to one NVLink
    multicast object: the target of the multicast fused GEMM + all-gather
    (bwgemm.gemm_*_allgather_multicast), whose multimem stores NVSwitch replicates into every
    rank's copy. Collective (every rank constructs it with the same shape). `available` is
    False where the platform offers no multicast (then `mc` is 0 and nothing may use it)."""

    def __init__(self, M: int, N_total: int, dtype, device, group=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.C = symm_mem.empty((M, N_total), dtype=dtype, device=device)
        self.handle = symm_mem.rendezvous(self.C, group if group is not None else dist.group.WORLD)
        self.mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        self.available = self.mc != 0
