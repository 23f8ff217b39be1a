"""The GEMM and quantiser entry points can be captured into a CUDA graph (after a first eager
call has done the one-time per-device set-up) and replayed: same bits as eager calls, except
for split-K problems (M <= 256), whose partial tiles are added in arrival order (FP32
reduction order differs from run to run; the values agree to rounding)."""
import numpy as np
import pytest

import bwgemm
import oracle as o

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (128, 4096, 2048), (4096, 4096, 512)])
def test_graph_replay_matches_eager(cuda_dev, M, N, K):
    import torch

    x_a = _t(o.seeded_normal((M, K), 11), cuda_dev)
    x_b = _t(o.seeded_normal((K, N), 12), cuda_dev)
    A16, B16 = x_a.half(), x_b.half()
    C16 = torch.empty((M, N), device=cuda_dev)
    qa = torch.empty((M, K), dtype=torch.uint8, device=cuda_dev)
    qb = torch.empty((N, K), dtype=torch.uint8, device=cuda_dev)
    sa = torch.empty(1, device=cuda_dev)
    sb = torch.empty(1, device=cuda_dev)
    C8 = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
    qma, sfa = bwgemm.quantize_mxfp4(x_a, False)
    qmb, sfb = bwgemm.quantize_mxfp4(x_b, True)
    C4 = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_dev)
    s = torch.cuda.Stream(cuda_dev)

    def work():
        bwgemm.gemm_f16(A16, B16, C16, stream=s)
        bwgemm.quantize_fp8(x_a, False, bwgemm.SCALE_AMAX, dst=qa, scale_out=sa, stream=s)
        bwgemm.quantize_fp8(x_b, True, bwgemm.SCALE_AMAX, dst=qb, scale_out=sb, stream=s)
        bwgemm.gemm_fp8(qa, qb, sa, sb, C8, stream=s)
        bwgemm.quantize_mxfp4(x_a, False, dst=qma, sf=sfa, stream=s)
        bwgemm.quantize_mxfp4(x_b, True, dst=qmb, sf=sfb, stream=s)
        bwgemm.gemm_mxfp4(qma, qmb, sfa, sfb, K, C=C4, stream=s)

    with torch.cuda.stream(s):
        work()  # eager: one-time set-up (device state, workspaces, kernel attributes)
    torch.cuda.synchronize()
    eager = [t.clone() for t in (C16, C8, C4)]
    for t in (C16, C8, C4):
        t.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        work()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert bwgemm.device_status() == 0
    split = M <= 256
    for got, want in zip((C16, C8, C4), eager):
        if split:
            assert torch.allclose(got.float(), want.float(), rtol=1e-5, atol=1e-4)
        else:
            assert torch.equal(got, want)
