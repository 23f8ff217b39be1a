"""GPU parity of the single-process sharded GEMM (bw_gemm_sharded): every shard's C against the
FP64 oracle over the same quantised inputs, and the gathered C against the shards it is made of
(bit-identical: the gather only moves bytes). Runs on one GPU (ngpu = 1) and, where the box has
more, over every visible GPU (up to 4) with the NCCL all-gather."""
import numpy as np
import pytest

import bwgemm
import oracle as o

pytestmark = pytest.mark.gpu


def _t(x, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _np(t):
    import torch

    return (t.float() if t.dtype == torch.bfloat16 else t).cpu().numpy()


def _devices(n):
    import torch

    return [torch.device(f"cuda:{i}") for i in range(n)]


def _ngpus():
    import torch

    return [1] + ([min(4, torch.cuda.device_count())] if torch.cuda.device_count() >= 2 else [])


def _sync_all(devs):
    import torch

    for d in devs:
        torch.cuda.synchronize(d)


@pytest.mark.parametrize("g", _ngpus())
def test_sharded_f16_gathered(cuda_dev, g):
    import torch

    M, N, K = 384, 256 * g, 512
    A = o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((M, K), 61)))
    B = o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((K, N), 62)))
    devs = _devices(g)
    ns = N // g
    parts = []
    for r, d in enumerate(devs):
        bwgemm.init(d.index)
        parts.append({"A": _t(A, d).half(), "B": _t(B[:, r * ns:(r + 1) * ns], d).half(),
                      "C": torch.empty((M, ns), device=d), "C_gathered": torch.empty((M, N), device=d)})
    bwgemm.gemm_sharded(bwgemm.DTYPE_F16, parts, M, N, K, bwgemm.OUT_F32, gather=True)
    _sync_all(devs)
    R = o.gemm_f64(A, B)
    tol = o.f16_tolerance(K, np.abs(A).max(), np.abs(B).max())
    shards = [_np(p["C"]) for p in parts]
    for r in range(g):
        assert np.abs(shards[r] - R[:, r * ns:(r + 1) * ns]).max() <= tol
    full = np.concatenate(shards, axis=1)
    for p in parts:
        assert np.array_equal(_np(p["C_gathered"]), full)
    torch.cuda.set_device(0)


@pytest.mark.parametrize("g", _ngpus())
@pytest.mark.parametrize("out", [bwgemm.OUT_F32, bwgemm.OUT_BF16])
def test_sharded_fp8_gathered(cuda_dev, g, out):
    import torch

    M, N, K = 256, 384 * g, 1024
    A = o.seeded_normal((M, K), 63)
    B = o.seeded_normal((K, N), 64)
    qa, sa = bwgemm.quantize_fp8(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX)
    qb, sb = bwgemm.quantize_fp8(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX)  # N x K, one scale for all shards
    torch.cuda.synchronize()
    devs = _devices(g)
    ns = N // g
    odt = torch.float32 if out == bwgemm.OUT_F32 else torch.bfloat16
    parts = []
    for r, d in enumerate(devs):
        bwgemm.init(d.index)
        parts.append({"A": qa.to(d), "B": qb[r * ns:(r + 1) * ns].contiguous().to(d), "scale_a": sa.to(d),
                      "scale_b": sb.to(d), "C": torch.empty((M, ns), dtype=odt, device=d),
                      "C_gathered": torch.empty((M, N), dtype=odt, device=d)})
    _sync_all(devs)
    bwgemm.gemm_sharded(bwgemm.DTYPE_FP8, parts, M, N, K, out, gather=True)
    _sync_all(devs)
    ra, rsa = o.quant_fp8(A, False, o.SCALE_AMAX)
    rb, rsb = o.quant_fp8(B, True, o.SCALE_AMAX)
    R = o.gemm_f64(o.dequant_fp8(ra), o.dequant_fp8(rb), b_trans=True) * np.float64(np.float32(rsa * rsb))
    da = o.dequant_fp8(ra) * np.float32(rsa)
    db = o.dequant_fp8(rb) * np.float32(rsb)
    tol = o.lowp_tolerance(K, np.abs(da).max(), np.abs(db).max(), np.abs(R).max(), out == bwgemm.OUT_BF16)
    shards = [_np(p["C"]) for p in parts]
    for r in range(g):
        assert np.abs(shards[r] - R[:, r * ns:(r + 1) * ns]).max() <= tol
    full = np.concatenate(shards, axis=1)
    for p in parts:
        assert np.array_equal(_np(p["C_gathered"]), full)
    torch.cuda.set_device(0)


@pytest.mark.parametrize("g", _ngpus())
def test_sharded_mxfp4_without_gather(cuda_dev, g):
    import torch

    M, N, K = 256, 256 * g, 512
    A = o.seeded_normal((M, K), 65)
    B = o.seeded_normal((K, N), 66)
    devs = _devices(g)
    ns = N // g
    parts = []
    for r, d in enumerate(devs):
        bwgemm.init(d.index)
        with torch.cuda.device(d):
            qa, sfa = bwgemm.quantize_mxfp4(_t(A, d), False, bwgemm.MX_BLOCK32)
            qb, sfb = bwgemm.quantize_mxfp4(_t(B[:, r * ns:(r + 1) * ns], d), True, bwgemm.MX_BLOCK32)
        parts.append({"A": qa, "B": qb, "sfA": sfa, "sfB": sfb,
                      "C": torch.empty((M, ns), dtype=torch.float32, device=d)})
    _sync_all(devs)
    bwgemm.gemm_sharded(bwgemm.DTYPE_MXFP4, parts, M, N, K, bwgemm.OUT_F32, gather=False)
    _sync_all(devs)
    ra, rsfa = o.quant_mxfp4(A, False, o.MX_BLOCK32)
    rb, rsfb = o.quant_mxfp4(B, True, o.MX_BLOCK32)
    da, db = o.dequant_mxfp4(ra, rsfa, K), o.dequant_mxfp4(rb, rsfb, K)
    R = o.gemm_f64(da, db, b_trans=True)
    tol = o.lowp_tolerance(K, np.abs(da).max(), np.abs(db).max())
    for r, p in enumerate(parts):
        assert np.abs(_np(p["C"]) - R[:, r * ns:(r + 1) * ns]).max() <= tol
    torch.cuda.set_device(0)
