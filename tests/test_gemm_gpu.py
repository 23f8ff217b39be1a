"""GPU parity: the tcgen05 GEMMs and device quantisers (through the C ABI) against the oracle.

Tolerances are the north star's:
  FP16:          max|C - C_ref| <= 2^-10 * sqrt(K) * max|a| * max|b|
  FP8/FP4/MXFP4: max|C - C_ref| <= 1e-5 * K * max|a_deq| * max|b_deq|  (+ 2^-8 |C_ref| for BF16 out)
where C_ref is the FP64 oracle GEMM over the identically quantised inputs. Quantisers are
bit-exact. Full-size (8192) shapes are checked through exactly representable inputs
(small integers: FP32 accumulation is exact) on sampled rows and columns.
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


def _f16(x):
    return o.f16_to_f32(o.f32_to_f16(x))


def _status_ok():
    assert bwgemm.device_status() == 0


F16_SHAPES = [(256, 256, 256), (1024, 1024, 1024), (129, 136, 72), (128, 8, 8), (1, 8, 64), (300, 520, 1000),
              (640, 1280, 2048), (4096, 256, 64)]


@pytest.mark.parametrize("M,N,K", F16_SHAPES)
@pytest.mark.parametrize("b_transposed", [False, True])
def test_f16_parity(cuda_dev, M, N, K, b_transposed):
    import torch

    A = _f16(o.seeded_uniform((M, K), 1))
    B = _f16(o.seeded_uniform((K, N), 2))
    Bdev = B.T.copy() if b_transposed else B
    C = bwgemm.gemm_f16(_t(A, cuda_dev).half(), _t(Bdev, cuda_dev).half(), b_transposed=b_transposed)
    torch.cuda.synchronize()
    _status_ok()
    R = o.gemm_f64(A, B)
    err = np.abs(_np(C) - R).max()
    tol = o.f16_tolerance(K, np.abs(A).max(), np.abs(B).max())
    assert err <= tol, (err, tol)


def test_f16_k_zero_and_empty(cuda_dev):
    import torch

    A = torch.zeros((64, 0), dtype=torch.float16, device=cuda_dev)
    B = torch.zeros((0, 64), dtype=torch.float16, device=cuda_dev)
    C = torch.full((64, 64), 7.0, device=cuda_dev)
    bwgemm.gemm_f16(A, B, C)
    assert float(C.abs().max()) == 0.0
    E = torch.empty((0, 64), dtype=torch.float32, device=cuda_dev)
    bwgemm.gemm_f16(torch.empty((0, 64), dtype=torch.float16, device=cuda_dev),
                    torch.empty((64, 64), dtype=torch.float16, device=cuda_dev), E)


def test_f16_rejects_bad_shapes(cuda_dev):
    import torch

    A = torch.zeros((64, 12), dtype=torch.float16, device=cuda_dev)
    B = torch.zeros((12, 64), dtype=torch.float16, device=cuda_dev)
    with pytest.raises(bwgemm.BwError) as e:
        bwgemm.gemm_f16(A, B)
    assert e.value.code == bwgemm.BW_ERR_INVALID


def _exact_ints(shape, seed, lo=-2, hi=2):
    return np.random.default_rng(seed).integers(lo, hi + 1, size=shape).astype(np.float32)


@pytest.mark.parametrize("M,N,K", [(8192, 8192, 8192), (16384, 2048, 8192), (128, 65536, 8192)])
def test_f16_full_size_exact(cuda_dev, M, N, K):
    """Integer inputs in [-2, 2]: every partial sum is exact in FP32, so the GPU result must
    equal the FP64 oracle bit for bit on the sampled rows and columns."""
    import torch

    A = _exact_ints((M, K), 11)
    B = _exact_ints((K, N), 12)
    C = _np(bwgemm.gemm_f16(_t(A, cuda_dev).half(), _t(B, cuda_dev).half()))
    torch.cuda.synchronize()
    _status_ok()
    rng = np.random.default_rng(3)
    rows = np.unique(np.concatenate([rng.integers(0, M, 48), [0, M - 1]]))
    cols = np.unique(np.concatenate([rng.integers(0, N, 48), [0, N - 1]]))
    Rr = o.gemm_f64(A[rows], B)
    assert np.array_equal(C[rows].astype(np.float64), Rr)
    Rc = o.gemm_f64(A, np.ascontiguousarray(B[:, cols]))
    assert np.array_equal(C[:, cols].astype(np.float64), Rc)


def test_f16_linearity_full_size(cuda_dev):
    """C(A, B1 + B2) == C(A, B1) + C(A, B2) on exactly representable inputs at 8192^3."""
    import torch

    M = N = K = 8192
    A = _t(_exact_ints((M, K), 21), cuda_dev).half()
    B1 = _t(_exact_ints((K, N), 22, -1, 1), cuda_dev).half()
    B2 = _t(_exact_ints((K, N), 23, -1, 1), cuda_dev).half()
    C12 = bwgemm.gemm_f16(A, (B1 + B2).contiguous())
    C1 = bwgemm.gemm_f16(A, B1)
    C2 = bwgemm.gemm_f16(A, B2)
    torch.cuda.synchronize()
    assert torch.equal(C12, C1 + C2)


# ------------------------------------------------------------------ quantisers
def test_quantisers_match_golden(cuda_dev):
    g = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "quant_golden.npz"))
    x = _t(g["x"], cuda_dev)
    q, s = bwgemm.quantize_fp8(x, False, bwgemm.SCALE_NONE)
    assert np.array_equal(_np(q), g["fp8"])
    q, s = bwgemm.quantize_fp4(x, False, bwgemm.SCALE_FIXED8, bwgemm.FP4_BYTE_SHL2)
    assert np.array_equal(_np(q), g["fp4_byte"])
    q, sf = bwgemm.quantize_mxfp4(x, False, bwgemm.MX_UNIT_FIXED8)
    assert np.array_equal(_np(q), g["mxfp4_ref"])
    q, sf = bwgemm.quantize_mxfp4(x, False, bwgemm.MX_BLOCK32)
    assert np.array_equal(_np(q), g["mxfp4_q"])
    assert np.array_equal(_np(sf), g["mxfp4_sf"])
    h = _np(bwgemm.quantize_f16(x).view(__import__("torch").int16)).view(np.uint16)
    nan = np.isnan(g["x"])  # NaN payloads may differ; both must be NaN codes
    assert np.array_equal(h[~nan], g["f16"][~nan])
    assert np.all((h[nan] & 0x7FFF) > 0x7C00) and np.all((g["f16"][nan] & 0x7FFF) > 0x7C00)


@pytest.mark.parametrize("transpose", [False, True])
@pytest.mark.parametrize("mode", [bwgemm.SCALE_NONE, bwgemm.SCALE_FIXED8, bwgemm.SCALE_AMAX])
@pytest.mark.parametrize("shape", [(200, 328), (256, 96), (4096, 160), (37, 45)])
def test_quantize_fp8_bit_exact(cuda_dev, transpose, mode, shape):
    """16-wide vector paths (rows % 16 == 0, n % 16 == 0) and the element-wise fallbacks."""
    x = o.seeded_normal(shape, 5) * 3
    q, s = bwgemm.quantize_fp8(_t(x, cuda_dev), transpose, mode)
    qr, sr = o.quant_fp8(x, transpose, mode)
    assert np.array_equal(_np(q), qr)
    assert float(_np(s)[0]) == sr


@pytest.mark.parametrize("transpose", [False, True])
@pytest.mark.parametrize("container", [bwgemm.FP4_PACKED, bwgemm.FP4_BYTE_SHL2])
@pytest.mark.parametrize("mode", [bwgemm.SCALE_FIXED8, bwgemm.SCALE_AMAX])
@pytest.mark.parametrize("shape", [(192, 256), (130, 66)])
def test_quantize_fp4_bit_exact(cuda_dev, transpose, container, mode, shape):
    x = o.seeded_normal(shape, 6)
    q, s = bwgemm.quantize_fp4(_t(x, cuda_dev), transpose, mode, container)
    qr, sr = o.quant_fp4(x, transpose, mode, container)
    assert np.array_equal(_np(q), qr)
    assert float(_np(s)[0]) == sr


@pytest.mark.parametrize("transpose", [False, True])
@pytest.mark.parametrize("mode", [bwgemm.MX_UNIT_FIXED8, bwgemm.MX_BLOCK32])
@pytest.mark.parametrize("shape", [(256, 320), (288, 96), (64, 1312), (4096, 512)])
def test_quantize_mxfp4_bit_exact(cuda_dev, transpose, mode, shape):
    """Ragged tails in both directions (K not a multiple of 128 or 256, outer not a multiple
    of 32 or 128), zero blocks, huge and non-finite values."""
    x = o.seeded_normal(shape, 7)
    x[:, :7] *= 1e3
    x[:32, :32] = 0.0
    x[40, 40] = np.float32(3e38)
    x[41, 41] = np.inf
    x[42, 42] = -np.inf
    x[43, 43] = np.nan
    x[44, 44] = np.float32(1e-42)
    q, sf = bwgemm.quantize_mxfp4(_t(x, cuda_dev), transpose, mode)
    qr, sfr = o.quant_mxfp4(x, transpose, mode)
    assert np.array_equal(_np(q), qr)
    assert np.array_equal(_np(sf), sfr)


# ------------------------------------------------------------------ low-precision GEMMs
LOWP_SHAPES = [(256, 256, 256), (1024, 1024, 1024), (129, 136, 96), (384, 640, 2048), (128, 8, 64)]


@pytest.mark.parametrize("M,N,K", LOWP_SHAPES)
@pytest.mark.parametrize("out", [bwgemm.OUT_F32, bwgemm.OUT_BF16])
def test_fp8_parity(cuda_dev, M, N, K, out):
    import torch

    if K % 16:
        pytest.skip("fp8 needs K % 16 == 0")
    A = o.seeded_normal((M, K), 31)
    B = o.seeded_normal((K, N), 32)
    qa, sa = bwgemm.quantize_fp8(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX)
    qb, sb = bwgemm.quantize_fp8(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX)
    C = _np(bwgemm.gemm_fp8(qa, qb, sa, sb, out_dtype=out))
    torch.cuda.synchronize()
    _status_ok()
    ra, rsa = o.quant_fp8(A, False, o.SCALE_AMAX)
    rb, rsb = o.quant_fp8(B, True, o.SCALE_AMAX)
    da = o.dequant_fp8(ra) * np.float32(rsa)
    db = o.dequant_fp8(rb) * np.float32(rsb)
    R = o.gemm_f64(o.dequant_fp8(ra), o.dequant_fp8(rb), b_trans=True) * (np.float64(np.float32(rsa * rsb)))
    tol = o.lowp_tolerance(K, np.abs(da).max(), np.abs(db).max(), np.abs(R).max(), out == bwgemm.OUT_BF16)
    err = np.abs(C - R).max()
    assert err <= tol, (err, tol)


@pytest.mark.parametrize("M,N,K", LOWP_SHAPES)
def test_mxfp4_parity(cuda_dev, M, N, K):
    import torch

    A = o.seeded_normal((M, K), 41)
    B = o.seeded_normal((K, N), 42)
    qa, sfa = bwgemm.quantize_mxfp4(_t(A, cuda_dev), False, bwgemm.MX_BLOCK32)
    qb, sfb = bwgemm.quantize_mxfp4(_t(B, cuda_dev), True, bwgemm.MX_BLOCK32)
    C = _np(bwgemm.gemm_mxfp4(qa, qb, sfa, sfb, K, out_dtype=bwgemm.OUT_F32))
    torch.cuda.synchronize()
    _status_ok()
    ra, rsfa = o.quant_mxfp4(A, False, o.MX_BLOCK32)
    rb, rsfb = o.quant_mxfp4(B, True, o.MX_BLOCK32)
    da = o.dequant_mxfp4(ra, rsfa, K)
    db = o.dequant_mxfp4(rb, rsfb, K)
    R = o.gemm_f64(da, db, b_trans=True)
    tol = o.lowp_tolerance(K, np.abs(da).max(), np.abs(db).max())
    err = np.abs(C - R).max()
    assert err <= tol, (err, tol)


@pytest.mark.parametrize("M,N,K", LOWP_SHAPES)
def test_fp4_per_tensor_parity(cuda_dev, M, N, K):
    import torch

    A = o.seeded_normal((M, K), 51)
    B = o.seeded_normal((K, N), 52)
    qa, sa = bwgemm.quantize_fp4(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX, bwgemm.FP4_PACKED)
    qb, sb = bwgemm.quantize_fp4(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX, bwgemm.FP4_PACKED)
    C = _np(bwgemm.gemm_fp4(qa, qb, K, sa, sb, out_dtype=bwgemm.OUT_BF16))
    torch.cuda.synchronize()
    _status_ok()
    ra, rsa = o.quant_fp4(A, False, o.SCALE_AMAX, o.FP4_PACKED)
    rb, rsb = o.quant_fp4(B, True, o.SCALE_AMAX, o.FP4_PACKED)
    da = o.dequant_mxfp4(ra, None, K)
    db = o.dequant_mxfp4(rb, None, K)
    R = o.gemm_f64(da, db, b_trans=True) * np.float64(np.float32(rsa) * np.float32(rsb))
    tol = o.lowp_tolerance(K, np.abs(da).max() * rsa, np.abs(db).max() * rsb, np.abs(R).max(), True)
    err = np.abs(C - R).max()
    assert err <= tol, (err, tol)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("M,N,world", [(64, 96, 4), (33, 72, 4), (5, 4096, 8)])
def test_unshard_columns(cuda_dev, dtype, M, N, world):
    """Both element sizes, 16-byte and scalar paths (72 / 4 columns per shard is not a whole
    number of 16-byte groups); a BF16 buffer must not be walked as FP32 (that read past its end)."""
    import torch

    full = o.seeded_uniform((M, N), 9)
    shards = np.stack([full[:, r * (N // world):(r + 1) * (N // world)] for r in range(world)])
    src = _t(np.ascontiguousarray(shards), cuda_dev).to(getattr(torch, dtype))
    out = bwgemm.unshard_columns(src, M, N, world)
    torch.cuda.synchronize()
    assert out.dtype == src.dtype
    assert torch.equal(out.cpu(), torch.from_numpy(full).to(src.dtype))
    with pytest.raises(ValueError):
        bwgemm.unshard_columns(src, M, N + world, world)


@pytest.mark.parametrize("kind", ["f16", "fp8"])
def test_pair_kernel_staged_epilogue_when_c_not_32b_aligned(cuda_dev, kind):
    """C only 16-byte aligned selects the shared-memory/TMA-store epilogue of the CTA-pair
    kernel instead of the direct 32-byte stores; results must be identical."""
    import torch

    M = N = K = 2048
    if kind == "f16":
        A = _f16(o.seeded_uniform((M, K), 61))
        B = _f16(o.seeded_uniform((K, N), 62))
        Ad, Bd = _t(A, cuda_dev).half(), _t(B, cuda_dev).half()
        ref = bwgemm.gemm_f16(Ad, Bd)
        buf = torch.empty(M * N + 4, dtype=torch.float32, device=cuda_dev)
        C = buf[4:].view(M, N)  # 16-byte offset from a 256-byte aligned base
        bwgemm.gemm_f16(Ad, Bd, C)
    else:
        qa, sa = bwgemm.quantize_fp8(_t(o.seeded_normal((M, K), 63), cuda_dev), False)
        qb, sb = bwgemm.quantize_fp8(_t(o.seeded_normal((K, N), 64), cuda_dev), True)
        ref = bwgemm.gemm_fp8(qa, qb, sa, sb)
        buf = torch.empty(M * N + 8, dtype=torch.bfloat16, device=cuda_dev)
        C = buf[8:].view(M, N)
        bwgemm.gemm_fp8(qa, qb, sa, sb, C)
    torch.cuda.synchronize()
    _status_ok()
    assert C.data_ptr() % 32 == 16
    assert torch.equal(C, ref)


MX_PAIR_SHAPES = [(512, 512, 512), (300, 520, 1024), (1024, 768, 800), (2048, 2048, 4096), (512, 1344, 512)]


@pytest.mark.parametrize("M,N,K", MX_PAIR_SHAPES)
@pytest.mark.parametrize("out", [bwgemm.OUT_F32, bwgemm.OUT_BF16])
@pytest.mark.parametrize("tn", ["192", "256"])
def test_mxfp4_pair_kernel_parity(cuda_dev, monkeypatch, M, N, K, out, tn):
    """The CTA-pair block-scaled kernel (forced with BW_PAIR=1) against the oracle, including
    M/N tails inside a 256 x 256 tile and K not a multiple of the 512-deep stage."""
    import torch

    monkeypatch.setenv("BW_PAIR", "1")
    monkeypatch.setenv("BW_MX_TN", tn)
    A = o.seeded_normal((M, K), 71)
    B = o.seeded_normal((K, N), 72)
    A[:, :5] *= 100.0  # a few blocks with large scales
    qa, sfa = bwgemm.quantize_mxfp4(_t(A, cuda_dev), False, bwgemm.MX_BLOCK32)
    qb, sfb = bwgemm.quantize_mxfp4(_t(B, cuda_dev), True, bwgemm.MX_BLOCK32)
    C = _np(bwgemm.gemm_mxfp4(qa, qb, sfa, sfb, K, out_dtype=out))
    torch.cuda.synchronize()
    _status_ok()
    ra, rsfa = o.quant_mxfp4(A, False, o.MX_BLOCK32)
    rb, rsfb = o.quant_mxfp4(B, True, o.MX_BLOCK32)
    da, db = o.dequant_mxfp4(ra, rsfa, K), o.dequant_mxfp4(rb, rsfb, K)
    R = o.gemm_f64(da, db, b_trans=True)
    tol = o.lowp_tolerance(K, np.abs(da).max(), np.abs(db).max(), np.abs(R).max(), out == bwgemm.OUT_BF16)
    assert np.abs(C - R).max() <= tol


@pytest.mark.parametrize("M,N,K", [(512, 512, 512), (300, 520, 1024), (1024, 2240, 2048)])
@pytest.mark.parametrize("out", [bwgemm.OUT_F32, bwgemm.OUT_BF16])
def test_fp4_pair_kernel_parity(cuda_dev, monkeypatch, M, N, K, out):
    import torch

    monkeypatch.setenv("BW_PAIR", "1")
    A = o.seeded_normal((M, K), 81)
    B = o.seeded_normal((K, N), 82)
    qa, sa = bwgemm.quantize_fp4(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX, bwgemm.FP4_PACKED)
    qb, sb = bwgemm.quantize_fp4(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX, bwgemm.FP4_PACKED)
    C = _np(bwgemm.gemm_fp4(qa, qb, K, sa, sb, out_dtype=out))
    torch.cuda.synchronize()
    _status_ok()
    ra, rsa = o.quant_fp4(A, False, o.SCALE_AMAX, o.FP4_PACKED)
    rb, rsb = o.quant_fp4(B, True, o.SCALE_AMAX, o.FP4_PACKED)
    da, db = o.dequant_mxfp4(ra, None, K), o.dequant_mxfp4(rb, None, K)
    R = o.gemm_f64(da, db, b_trans=True) * np.float64(np.float32(rsa) * np.float32(rsb))
    tol = o.lowp_tolerance(K, np.abs(da).max() * rsa, np.abs(db).max() * rsb, np.abs(R).max(),
                           out == bwgemm.OUT_BF16)
    assert np.abs(C - R).max() <= tol


@pytest.mark.parametrize("M,N,K", [(128, 4096, 1024), (77, 2056, 528), (200, 1024, 4096), (1, 1024, 1024)])
@pytest.mark.parametrize("kind", ["f16", "fp8", "fp8_bf16"])
@pytest.mark.parametrize("splits", ["2", "3", "8"])
def test_splitk_parity(cuda_dev, monkeypatch, M, N, K, kind, splits):
    """Split-K (partial tiles TMA-reduce-added into zeroed C, or for BF16 C into an FP32
    workspace converted afterwards), forced with BW_SPLITK; uneven k-slab ranges and more
    splits than k-slabs included."""
    import torch

    monkeypatch.setenv("BW_SPLITK", splits)
    if kind == "f16":
        A = _f16(o.seeded_uniform((M, K), 91))
        B = _f16(o.seeded_uniform((K, N), 92))
        C = _np(bwgemm.gemm_f16(_t(A, cuda_dev).half(), _t(B, cuda_dev).half()))
        R = o.gemm_f64(A, B)
        tol = o.f16_tolerance(K, np.abs(A).max(), np.abs(B).max())
    else:
        if K % 16:
            pytest.skip("fp8 needs K % 16 == 0")
        A = o.seeded_normal((M, K), 93)
        B = o.seeded_normal((K, N), 94)
        qa, sa = bwgemm.quantize_fp8(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX)
        qb, sb = bwgemm.quantize_fp8(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX)
        bf16 = kind == "fp8_bf16"
        C = _np(bwgemm.gemm_fp8(qa, qb, sa, sb, out_dtype=bwgemm.OUT_BF16 if bf16 else bwgemm.OUT_F32))
        ra, rsa = o.quant_fp8(A, False, o.SCALE_AMAX)
        rb, rsb = o.quant_fp8(B, True, o.SCALE_AMAX)
        R = o.gemm_f64(o.dequant_fp8(ra), o.dequant_fp8(rb), b_trans=True) * float(np.float32(rsa) * np.float32(rsb))
        tol = o.lowp_tolerance(K, 448 * rsa, 448 * rsb, np.abs(R).max(), bf16)
    torch.cuda.synchronize()
    _status_ok()
    assert np.abs(C - R).max() <= tol


def test_splitk_bf16_workspace_per_stream(cuda_dev):
    """Two streams running split-K BF16 GEMMs at once use separate FP32 workspaces; a larger
    problem afterwards grows the workspace."""
    import torch

    outs, refs = [], []
    streams = [torch.cuda.Stream(cuda_dev), torch.cuda.Stream(cuda_dev)]
    for i, (M, N, K) in enumerate([(128, 8192, 4096), (64, 4096, 8192)]):
        A = o.seeded_normal((M, K), 121 + i)
        B = o.seeded_normal((K, N), 131 + i)
        qa, sa = bwgemm.quantize_fp8(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX)
        qb, sb = bwgemm.quantize_fp8(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX)
        torch.cuda.synchronize()
        ra, rsa = o.quant_fp8(A, False, o.SCALE_AMAX)
        rb, rsb = o.quant_fp8(B, True, o.SCALE_AMAX)
        R = o.gemm_f64(o.dequant_fp8(ra), o.dequant_fp8(rb), b_trans=True) * float(np.float32(rsa) * np.float32(rsb))
        refs.append((R, o.lowp_tolerance(K, 448 * rsa, 448 * rsb, np.abs(R).max(), True)))
        outs.append((qa, qb, sa, sb))
    Cs = []
    for _ in range(3):
        Cs = [bwgemm.gemm_fp8(*outs[i], out_dtype=bwgemm.OUT_BF16, stream=streams[i]) for i in range(2)]
    torch.cuda.synchronize()
    _status_ok()
    for C, (R, tol) in zip(Cs, refs):
        assert np.abs(_np(C) - R).max() <= tol
    # growth: a wider problem on the first stream
    M, N, K = 256, 16384, 2048
    A = o.seeded_normal((M, K), 141)
    B = o.seeded_normal((K, N), 142)
    qa, sa = bwgemm.quantize_fp8(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX)
    qb, sb = bwgemm.quantize_fp8(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX)
    C = bwgemm.gemm_fp8(qa, qb, sa, sb, out_dtype=bwgemm.OUT_BF16, stream=streams[0])
    torch.cuda.synchronize()
    ra, rsa = o.quant_fp8(A, False, o.SCALE_AMAX)
    rb, rsb = o.quant_fp8(B, True, o.SCALE_AMAX)
    R = o.gemm_f64(o.dequant_fp8(ra), o.dequant_fp8(rb), b_trans=True) * float(np.float32(rsa) * np.float32(rsb))
    assert np.abs(_np(C) - R).max() <= o.lowp_tolerance(K, 448 * rsa, 448 * rsb, np.abs(R).max(), True)


@pytest.mark.parametrize("M,N,K", [(512, 1024, 512), (300, 1040, 320), (256, 512, 64), (1024, 2064, 1024)])
@pytest.mark.parametrize("kind", ["f16", "fp8_f32", "fp8_bf16"])
def test_wide_pair_kernel_parity(cuda_dev, monkeypatch, M, N, K, kind):
    """The 256 x 512 CTA-pair kernel (two N halves released separately) against the oracle,
    ragged M / N / K edges included."""
    import torch

    monkeypatch.setenv("BW_PAIR", "1")
    monkeypatch.setenv("BW_WIDE", "1")
    if kind == "f16":
        A = _f16(o.seeded_uniform((M, K), 111))
        B = _f16(o.seeded_uniform((K, N), 112))
        C = _np(bwgemm.gemm_f16(_t(A, cuda_dev).half(), _t(B, cuda_dev).half()))
        torch.cuda.synchronize()
        _status_ok()
        tol = o.f16_tolerance(K, np.abs(A).max(), np.abs(B).max())
        assert np.abs(C - o.gemm_f64(A, B)).max() <= tol
        return
    out = bwgemm.OUT_F32 if kind == "fp8_f32" else bwgemm.OUT_BF16
    A = o.seeded_normal((M, K), 113)
    B = o.seeded_normal((K, N), 114)
    qa, sa = bwgemm.quantize_fp8(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX)
    qb, sb = bwgemm.quantize_fp8(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX)
    C = _np(bwgemm.gemm_fp8(qa, qb, sa, sb, out_dtype=out))
    torch.cuda.synchronize()
    _status_ok()
    ra, rsa = o.quant_fp8(A, False, o.SCALE_AMAX)
    rb, rsb = o.quant_fp8(B, True, o.SCALE_AMAX)
    R = o.gemm_f64(o.dequant_fp8(ra), o.dequant_fp8(rb), b_trans=True) * float(np.float32(rsa) * np.float32(rsb))
    tol = o.lowp_tolerance(K, 448 * rsa, 448 * rsb, np.abs(R).max(), out == bwgemm.OUT_BF16)
    assert np.abs(C - R).max() <= tol


@pytest.mark.parametrize("N", [520, 1032])
def test_fp8_pair_bf16_out_with_unaligned_row_pitch(cuda_dev, monkeypatch, N):
    """N % 16 == 8 makes BF16 rows 16- but not 32-byte aligned: the pair kernel must take the
    staged epilogue, not the 32-byte direct stores."""
    import torch

    monkeypatch.setenv("BW_PAIR", "1")
    M, K = 512, 512
    A = o.seeded_normal((M, K), 101)
    B = o.seeded_normal((K, N), 102)
    qa, sa = bwgemm.quantize_fp8(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX)
    qb, sb = bwgemm.quantize_fp8(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX)
    C = _np(bwgemm.gemm_fp8(qa, qb, sa, sb, out_dtype=bwgemm.OUT_BF16))
    torch.cuda.synchronize()
    _status_ok()
    ra, rsa = o.quant_fp8(A, False, o.SCALE_AMAX)
    rb, rsb = o.quant_fp8(B, True, o.SCALE_AMAX)
    R = o.gemm_f64(o.dequant_fp8(ra), o.dequant_fp8(rb), b_trans=True) * float(np.float32(rsa) * np.float32(rsb))
    tol = o.lowp_tolerance(K, 448 * rsa, 448 * rsb, np.abs(R).max(), True)
    assert np.abs(C - R).max() <= tol


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 1024), (4096, 4096, 2048)])
def test_mxfp4_bit_identical_to_library(cuda_dev, M, N, K):
    """Independent check of the block-scaled path: the library MXFP4 GEMM that
    torch.nn.functional.scaled_mm runs (BlockWise1x32 with the 32x4x4-swizzled UE8M0 layout,
    which is our scale-factor layout; a CUTLASS kernel in this torch build - cuBLASLt 12.9
    rejects the E2M1 / VEC32_UE8M0 / BF16 combination) on the very same quantised buffers gives
    the same BF16 bits."""
    import torch

    F = torch.nn.functional
    if not hasattr(F, "scaled_mm") or not hasattr(torch, "float4_e2m1fn_x2"):
        pytest.skip("torch build without block-scaled FP4 scaled_mm")
    A = torch.randn(M, K, device=cuda_dev)
    B = torch.randn(K, N, device=cuda_dev)
    qa, sfa = bwgemm.quantize_mxfp4(A, False, bwgemm.MX_BLOCK32)
    qb, sfb = bwgemm.quantize_mxfp4(B, True, bwgemm.MX_BLOCK32)
    ours = bwgemm.gemm_mxfp4(qa, qb, sfa, sfb, K, out_dtype=bwgemm.OUT_BF16)
    lib = F.scaled_mm(qa.view(torch.float4_e2m1fn_x2), qb.view(torch.float4_e2m1fn_x2).t(),
                      sfa.view(torch.float8_e8m0fnu), F.ScalingType.BlockWise1x32,
                      sfb.view(torch.float8_e8m0fnu), F.ScalingType.BlockWise1x32,
                      swizzle_a=F.SwizzleType.SWIZZLE_32_4_4, swizzle_b=F.SwizzleType.SWIZZLE_32_4_4,
                      output_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    _status_ok()
    assert torch.equal(ours, lib)


@pytest.mark.parametrize("M,N,K", [(128, 4096, 1024), (77, 2056, 528), (200, 1024, 4096), (1, 1024, 1024),
                                   (256, 4104, 1024), (128, 16384, 2048), (64, 9216, 512), (129, 8192, 1024),
                                   (256, 40960, 512)])
@pytest.mark.parametrize("kind", ["f16", "f16_bt", "fp8", "fp8_bf16"])
def test_panel_kernel_parity(cuda_dev, monkeypatch, M, N, K, kind):
    """The column-panel kernel for short-and-wide problems (forced with BW_PANEL=1): panel
    widths from 32 to 512 columns (two MMAs per k-step above 256), one or two 128-row blocks of
    M per panel (M > 128), more panels than SMs (two waves), ragged M / N / K, both B layouts of
    FP16, FP32 and BF16 C."""
    import torch

    monkeypatch.setenv("BW_PANEL", "1")
    if kind.startswith("f16"):
        A = _f16(o.seeded_uniform((M, K), 151))
        B = _f16(o.seeded_uniform((K, N), 152))
        bt = kind == "f16_bt"
        C = _np(bwgemm.gemm_f16(_t(A, cuda_dev).half(), _t(B.T.copy() if bt else B, cuda_dev).half(),
                                b_transposed=bt))
        R = o.gemm_f64(A, B)
        tol = o.f16_tolerance(K, np.abs(A).max(), np.abs(B).max())
    else:
        A = o.seeded_normal((M, K), 153)
        B = o.seeded_normal((K, N), 154)
        qa, sa = bwgemm.quantize_fp8(_t(A, cuda_dev), False, bwgemm.SCALE_AMAX)
        qb, sb = bwgemm.quantize_fp8(_t(B, cuda_dev), True, bwgemm.SCALE_AMAX)
        bf16 = kind == "fp8_bf16"
        C = _np(bwgemm.gemm_fp8(qa, qb, sa, sb, out_dtype=bwgemm.OUT_BF16 if bf16 else bwgemm.OUT_F32))
        ra, rsa = o.quant_fp8(A, False, o.SCALE_AMAX)
        rb, rsb = o.quant_fp8(B, True, o.SCALE_AMAX)
        R = o.gemm_f64(o.dequant_fp8(ra), o.dequant_fp8(rb), b_trans=True) * float(np.float32(rsa) * np.float32(rsb))
        tol = o.lowp_tolerance(K, 448 * rsa, 448 * rsb, np.abs(R).max(), bf16)
    torch.cuda.synchronize()
    _status_ok()
    assert np.abs(C - R).max() <= tol
