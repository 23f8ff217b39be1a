"""GPU parity at the benchmark configurations themselves, with their own input distributions.

  FP16  8192^3   A, B ~ uniform[-1, 1] (seeded) rounded to FP16, FP32 accumulate, FP32 C
  FP8   8192^3   A, B ~ N(0, 1), E4M3 with a per-tensor scale amax/448, BF16 C
  MXFP4 8192^3   A, B ~ N(0, 1), E2M1 with one UE8M0 exponent per 32 K (floor(log2 amax) - 2), BF16 C
  FP4   8192^3   A, B ~ N(0, 1), E2M1 with a per-tensor scale amax/6, BF16 C
  shard 16384 x 8192 x 8192   one GPU's column shard of the 16384 x 65536 x 8192 sharded GEMM
                              at 8 GPUs (FP16 -> FP32 and FP8 -> BF16)
  skinny 128 x 65536 x 8192   the decode-style shape (split-K path), FP16 -> FP32, FP8 -> BF16

The device quantisers' codes and scales must equal the oracle's byte for byte over the whole
tensors; the GEMM output is compared with the FP64 oracle GEMM of the identically quantised
(dequantised) inputs on sampled rows (all N) and sampled columns (all M) - every row for the
skinny shape - under the north-star bounds:
  FP16:          max|C - C_ref| <= 2^-10 * sqrt(K) * max|a| * max|b|
  FP8/FP4/MXFP4: max|C - C_ref| <= 1e-5 * K * max|a_deq| * max|b_deq|  + 2^-8 |C_ref| (BF16 C)
A second, element-wise bound catches what the loose one lets through (a wrong small element
next to large ones): every element's error must stay within its own output rounding
(2^-8 |C_ref| for BF16, 2^-22 |C_ref| for FP32) plus an FP32 accumulation allowance of
2^-20 * K * max|a| * max|b|.
"""
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

    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.cpu().numpy()


def _samples(n, seed, count=64):
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([rng.choice(n, size=min(count, n), replace=False), [0, n - 1]]))


def _f16(x):
    return o.f16_to_f32(o.f32_to_f16(x))


def _check_sampled(C, dA, dB, b_trans, tol, tight, scale=1.0, seed=0, all_rows=False):
    """C (M x N, numpy) against FP64 dA x dB (x scale) on sampled rows and columns."""
    M, N = C.shape
    rows = np.arange(M) if all_rows else _samples(M, 100 + seed)
    Rr = o.gemm_f64(dA[rows], dB, b_trans=b_trans) * scale
    err_r = np.abs(C[rows].astype(np.float64) - Rr)
    assert err_r.max() <= tol, ("rows", err_r.max(), tol)
    assert np.all(err_r <= tight(Rr)), ("rows, tight bound", (err_r - tight(Rr)).max())
    if all_rows:
        return err_r.max()
    cols = _samples(N, 200 + seed)
    dBc = dB[cols] if b_trans else np.ascontiguousarray(dB[:, cols])
    Rc = o.gemm_f64(dA, dBc, b_trans=b_trans) * scale
    err_c = np.abs(C[:, cols].astype(np.float64) - Rc)
    assert err_c.max() <= tol, ("cols", err_c.max(), tol)
    assert np.all(err_c <= tight(Rc)), ("cols, tight bound", (err_c - tight(Rc)).max())
    return max(err_r.max(), err_c.max())


def _accum_slack(K, amax_a, amax_b):
    # FP32 accumulation error allowance: 2^-20 relative to the largest possible |C| (K products
    # of magnitude <= amax_a * amax_b), i.e. 16 FP32 ulps of that bound
    return 2.0 ** -20 * K * amax_a * amax_b


@pytest.mark.parametrize("M,N,K", [(8192, 8192, 8192), (16384, 8192, 8192), (128, 65536, 8192)],
                         ids=["headline_8192", "shard_16384x8192x8192", "skinny_128x65536x8192"])
def test_f16_config_uniform_inputs(cuda_dev, M, N, K):
    import torch

    A = _f16(o.seeded_uniform((M, K), 1001))
    B = _f16(o.seeded_uniform((K, N), 1002))
    C = _np(bwgemm.gemm_f16(_t(A, cuda_dev).half(), _t(B, cuda_dev).half()))
    torch.cuda.synchronize()
    assert bwgemm.device_status() == 0
    tol = o.f16_tolerance(K, np.abs(A).max(), np.abs(B).max())
    slack = _accum_slack(K, np.abs(A).max(), np.abs(B).max())
    _check_sampled(C, A, B, False, tol, lambda R: 2.0 ** -22 * np.abs(R) + slack, seed=M, all_rows=(M <= 128))


def _fp8_operands(M, N, K, dev, seed):
    A = o.seeded_normal((M, K), seed)
    B = o.seeded_normal((K, N), seed + 1)
    qa, sa = bwgemm.quantize_fp8(_t(A, dev), False, bwgemm.SCALE_AMAX)
    qb, sb = bwgemm.quantize_fp8(_t(B, dev), True, bwgemm.SCALE_AMAX)
    ra, rsa = o.quant_fp8(A, False, o.SCALE_AMAX)
    rb, rsb = o.quant_fp8(B, True, o.SCALE_AMAX)
    assert float(_np(sa)[0]) == rsa and float(_np(sb)[0]) == rsb
    assert np.array_equal(_np(qa), ra) and np.array_equal(_np(qb), rb)
    assert np.isclose(rsa, np.abs(A).max() / 448.0, rtol=1e-6)  # amax / 448
    return (qa, qb, sa, sb), (o.dequant_fp8(ra), o.dequant_fp8(rb), rsa, rsb)


@pytest.mark.parametrize("M,N,K", [(8192, 8192, 8192), (16384, 8192, 8192), (128, 65536, 8192)],
                         ids=["headline_8192", "shard_16384x8192x8192", "skinny_128x65536x8192"])
def test_fp8_config_amax448_bf16_out(cuda_dev, M, N, K):
    import torch

    (qa, qb, sa, sb), (da, db, rsa, rsb) = _fp8_operands(M, N, K, cuda_dev, 2001)
    C = _np(bwgemm.gemm_fp8(qa, qb, sa, sb, out_dtype=bwgemm.OUT_BF16))
    torch.cuda.synchronize()
    assert bwgemm.device_status() == 0
    scale = float(np.float32(rsa) * np.float32(rsb))
    ma, mb = np.abs(da).max() * rsa, np.abs(db).max() * rsb
    tol = o.lowp_tolerance(K, ma, mb) + 2.0 ** -8 * np.abs(C).max()
    slack = _accum_slack(K, ma, mb)
    _check_sampled(C, da, db, True, tol,
                   lambda R: 2.0 ** -8 * np.abs(R) + slack, scale=scale, seed=M, all_rows=(M <= 128))


def test_mxfp4_config_block32_bf16_out(cuda_dev):
    import torch

    M = N = K = 8192
    A = o.seeded_normal((M, K), 3001)
    B = o.seeded_normal((K, N), 3002)
    qa, sfa = bwgemm.quantize_mxfp4(_t(A, cuda_dev), False, bwgemm.MX_BLOCK32)
    qb, sfb = bwgemm.quantize_mxfp4(_t(B, cuda_dev), True, bwgemm.MX_BLOCK32)
    C = _np(bwgemm.gemm_mxfp4(qa, qb, sfa, sfb, K, out_dtype=bwgemm.OUT_BF16))
    torch.cuda.synchronize()
    assert bwgemm.device_status() == 0
    ra, rsfa = o.quant_mxfp4(A, False, o.MX_BLOCK32)
    rb, rsfb = o.quant_mxfp4(B, True, o.MX_BLOCK32)
    assert np.array_equal(_np(qa), ra) and np.array_equal(_np(sfa), rsfa)
    assert np.array_equal(_np(qb), rb) and np.array_equal(_np(sfb), rsfb)
    da, db = o.dequant_mxfp4(ra, rsfa, K), o.dequant_mxfp4(rb, rsfb, K)
    ma, mb = np.abs(da).max(), np.abs(db).max()
    tol = o.lowp_tolerance(K, ma, mb) + 2.0 ** -8 * np.abs(C).max()
    slack = _accum_slack(K, ma, mb)
    _check_sampled(C, da, db, True, tol, lambda R: 2.0 ** -8 * np.abs(R) + slack, seed=3)


def test_fp4_config_per_tensor_bf16_out(cuda_dev):
    import torch

    M = N = K = 8192
    A = o.seeded_normal((M, K), 4001)
    B = o.seeded_normal((K, N), 4002)
    qa, sa = bwgemm.quantize_fp4(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX, bwgemm.FP4_PACKED)
    qb, sb = bwgemm.quantize_fp4(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX, bwgemm.FP4_PACKED)
    C = _np(bwgemm.gemm_fp4(qa, qb, K, sa, sb, out_dtype=bwgemm.OUT_BF16))
    torch.cuda.synchronize()
    assert bwgemm.device_status() == 0
    ra, rsa = o.quant_fp4(A, False, o.SCALE_AMAX, o.FP4_PACKED)
    rb, rsb = o.quant_fp4(B, True, o.SCALE_AMAX, o.FP4_PACKED)
    assert np.array_equal(_np(qa), ra) and np.array_equal(_np(qb), rb)
    assert float(_np(sa)[0]) == rsa and np.isclose(rsa, np.abs(A).max() / 6.0, rtol=1e-6)  # amax / 6
    da, db = o.dequant_mxfp4(ra, None, K), o.dequant_mxfp4(rb, None, K)
    scale = float(np.float32(rsa) * np.float32(rsb))
    ma, mb = np.abs(da).max() * rsa, np.abs(db).max() * rsb
    tol = o.lowp_tolerance(K, ma, mb) + 2.0 ** -8 * np.abs(C).max()
    slack = _accum_slack(K, ma, mb)
    _check_sampled(C, da, db, True, tol, lambda R: 2.0 ** -8 * np.abs(R) + slack, scale=scale, seed=4)
