"""Randomised shapes through every dispatch path (pair / single-CTA / split-K / block-scaled,
FP32 and BF16 C, forced and automatic variants) against the oracle, with guard bands around C.
Seeded: the same shapes every run."""
import numpy as np
import pytest

import bwgemm
import oracle as o

pytestmark = pytest.mark.gpu

GUARD = 1024


def _shapes(seed, n, kmult):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        M = int(rng.integers(1, 700))
        N = int(rng.integers(1, 90)) * 16
        K = int(rng.integers(1, 40)) * kmult
        out.append((M, N, K))
    return out


def _t(x, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _guarded_c(M, N, dtype, dev):
    import torch

    elem = torch.empty((), dtype=dtype).element_size()
    whole = torch.full((GUARD * 2 + M * N * elem,), 0x5A, dtype=torch.uint8, device=dev)
    return whole, whole[GUARD:GUARD + M * N * elem].view(dtype).view(M, N)


def _guards_ok(whole, M, N, elem):
    w = whole.cpu().numpy()
    return (w[:GUARD] == 0x5A).all() and (w[GUARD + M * N * elem:] == 0x5A).all()


ENVS = [{}, {"BW_PAIR": "1"}, {"BW_PAIR": "0"}, {"BW_SPLITK": "4"}, {"BW_PAIR": "1", "BW_EPI_DIRECT": "0"},
        {"BW_PAIR": "1", "BW_WIDE": "1"}]


@pytest.mark.parametrize("case", range(12))
def test_fuzz_f16(cuda_dev, monkeypatch, case):
    import torch

    M, N, K = _shapes(1000 + case, 1, 16)[0]
    for k, v in ENVS[case % len(ENVS)].items():
        monkeypatch.setenv(k, v)
    A = o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((M, K), 2 * case + 1)))
    B = o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((K, N), 2 * case + 2)))
    whole, C = _guarded_c(M, N, torch.float32, cuda_dev)
    bwgemm.gemm_f16(_t(A, cuda_dev).half(), _t(B, cuda_dev).half(), C)
    torch.cuda.synchronize()
    assert bwgemm.device_status() == 0
    assert _guards_ok(whole, M, N, 4), (M, N, K)
    tol = o.f16_tolerance(K, np.abs(A).max(), np.abs(B).max())
    assert np.abs(C.cpu().numpy() - o.gemm_f64(A, B)).max() <= tol, (M, N, K)


@pytest.mark.parametrize("case", range(12))
@pytest.mark.parametrize("out", [bwgemm.OUT_F32, bwgemm.OUT_BF16])
def test_fuzz_fp8(cuda_dev, monkeypatch, case, out):
    import torch

    M, N, K = _shapes(2000 + case, 1, 16)[0]
    for k, v in ENVS[case % len(ENVS)].items():
        monkeypatch.setenv(k, v)
    A = o.seeded_normal((M, K), 3 * case + 1)
    B = o.seeded_normal((K, N), 3 * case + 2)
    qa, sa = bwgemm.quantize_fp8(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX)
    qb, sb = bwgemm.quantize_fp8(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX)
    dt = torch.float32 if out == bwgemm.OUT_F32 else torch.bfloat16
    whole, C = _guarded_c(M, N, dt, cuda_dev)
    bwgemm.gemm_fp8(qa, qb, sa, sb, C, out_dtype=out)
    torch.cuda.synchronize()
    assert bwgemm.device_status() == 0
    assert _guards_ok(whole, M, N, 4 if out == bwgemm.OUT_F32 else 2), (M, N, K)
    ra, rsa = o.quant_fp8(A, False, o.SCALE_AMAX)
    rb, rsb = o.quant_fp8(B, True, o.SCALE_AMAX)
    R = o.gemm_f64(o.dequant_fp8(ra), o.dequant_fp8(rb), b_trans=True) * float(np.float32(rsa) * np.float32(rsb))
    tol = o.lowp_tolerance(K, 448 * rsa, 448 * rsb, np.abs(R).max(), out == bwgemm.OUT_BF16)
    assert np.abs(C.float().cpu().numpy() - R).max() <= tol, (M, N, K)


@pytest.mark.parametrize("case", range(10))
def test_fuzz_mxfp4(cuda_dev, monkeypatch, case):
    import torch

    M, N, K = _shapes(3000 + case, 1, 32)[0]
    env = [{}, {"BW_PAIR": "1"}, {"BW_MX_PAIR": "0"}, {"BW_PAIR": "1", "BW_MX_TN": "192"}][case % 4]
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    A = o.seeded_normal((M, K), 5 * case + 1)
    B = o.seeded_normal((K, N), 5 * case + 2)
    qa, sfa = bwgemm.quantize_mxfp4(_t(A, cuda_dev), False, bwgemm.MX_BLOCK32)
    qb, sfb = bwgemm.quantize_mxfp4(_t(B, cuda_dev), True, bwgemm.MX_BLOCK32)
    whole, C = _guarded_c(M, N, torch.bfloat16, cuda_dev)
    bwgemm.gemm_mxfp4(qa, qb, sfa, sfb, K, C=C)
    torch.cuda.synchronize()
    assert bwgemm.device_status() == 0
    assert _guards_ok(whole, M, N, 2), (M, N, K)
    ra, rsfa = o.quant_mxfp4(A, False, o.MX_BLOCK32)
    rb, rsfb = o.quant_mxfp4(B, True, o.MX_BLOCK32)
    da, db = o.dequant_mxfp4(ra, rsfa, K), o.dequant_mxfp4(rb, rsfb, K)
    R = o.gemm_f64(da, db, b_trans=True)
    tol = o.lowp_tolerance(K, np.abs(da).max(), np.abs(db).max(), np.abs(R).max(), True)
    assert np.abs(C.float().cpu().numpy() - R).max() <= tol, (M, N, K)
