"""Out-of-bounds write checks (compute-sanitizer is closed on this pool): every output buffer
sits inside a larger allocation whose guard bands before and after hold a fixed bit pattern;
after the call the bands must be untouched. Ragged shapes reach every tile-edge path: the
CTA-pair kernel (direct and staged epilogues), the single-CTA kernel, split-K, the
block-scaled kernel and the quantisers."""
import numpy as np
import pytest

import bwgemm
import oracle as o

pytestmark = pytest.mark.gpu

GUARD = 4096  # bytes before and after
PATTERN = 0x5A


def _guarded(nbytes, dev, offset=0):
    """A uint8 buffer with guard bands; returns (whole, view_start) where the payload starts at
    GUARD + offset bytes (offset keeps the payload 16- or 32-byte aligned as needed)."""
    import torch

    whole = torch.full((GUARD + offset + nbytes + GUARD,), PATTERN, dtype=torch.uint8, device=dev)
    return whole, GUARD + offset


def _payload(whole, start, nbytes, dtype, shape):
    return whole[start:start + nbytes].view(dtype).view(shape)


def _check(whole, start, nbytes):
    import torch

    torch.cuda.synchronize()
    assert bwgemm.device_status() == 0
    before = whole[:start].cpu().numpy()
    after = whole[start + nbytes:].cpu().numpy()
    assert (before == PATTERN).all(), f"write before the buffer at {np.nonzero(before != PATTERN)[0][:4]}"
    assert (after == PATTERN).all(), f"write past the buffer at {np.nonzero(after != PATTERN)[0][:4]}"


def _t(x, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


SHAPES = [(129, 136, 72), (300, 520, 1000), (1000, 1032, 256), (77, 2056, 528)]
ENVS = [{}, {"BW_PAIR": "1"}, {"BW_PAIR": "1", "BW_EPI_DIRECT": "0"}, {"BW_PAIR": "0"}, {"BW_SPLITK": "3"},
        {"BW_PAIR": "1", "BW_WIDE": "1"}]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("env", ENVS, ids=["auto", "pair", "pair_staged", "single", "splitk", "pair_wide"])
def test_f16_writes_stay_inside_c(cuda_dev, monkeypatch, M, N, K, env):
    import torch

    for k, v in env.items():
        monkeypatch.setenv(k, v)
    A = _t(o.seeded_uniform((M, K), 1), cuda_dev).half()
    B = _t(o.seeded_uniform((K, N), 2), cuda_dev).half()
    nbytes = M * N * 4
    whole, start = _guarded(nbytes, cuda_dev)
    C = _payload(whole, start, nbytes, torch.float32, (M, N))
    bwgemm.gemm_f16(A, B, C)
    _check(whole, start, nbytes)


@pytest.mark.parametrize("M,N,K", [(129, 136, 96), (300, 528, 1024), (1000, 1040, 256)])
@pytest.mark.parametrize("out", [bwgemm.OUT_F32, bwgemm.OUT_BF16])
@pytest.mark.parametrize("env", ENVS, ids=["auto", "pair", "pair_staged", "single", "splitk", "pair_wide"])
def test_fp8_writes_stay_inside_c(cuda_dev, monkeypatch, M, N, K, out, env):
    import torch

    for k, v in env.items():
        monkeypatch.setenv(k, v)
    qa, sa = bwgemm.quantize_fp8(_t(o.seeded_normal((M, K), 3), cuda_dev), False, bwgemm.SCALE_AMAX)
    qb, sb = bwgemm.quantize_fp8(_t(o.seeded_normal((K, N), 4), cuda_dev), True, bwgemm.SCALE_AMAX)
    elem = 4 if out == bwgemm.OUT_F32 else 2
    nbytes = M * N * elem
    whole, start = _guarded(nbytes, cuda_dev)
    C = _payload(whole, start, nbytes, torch.float32 if elem == 4 else torch.bfloat16, (M, N))
    bwgemm.gemm_fp8(qa, qb, sa, sb, C, out_dtype=out)
    _check(whole, start, nbytes)


@pytest.mark.parametrize("M,N,K", [(129, 136, 96), (300, 520, 1024), (600, 1032, 512)])
@pytest.mark.parametrize("env", [{}, {"BW_PAIR": "1"}, {"BW_PAIR": "1", "BW_MX_TN": "192"}, {"BW_MX_PAIR": "0"}],
                         ids=["auto", "pair", "pair192", "single"])
def test_mxfp4_writes_stay_inside_c(cuda_dev, monkeypatch, M, N, K, env):
    import torch

    for k, v in env.items():
        monkeypatch.setenv(k, v)
    qa, sfa = bwgemm.quantize_mxfp4(_t(o.seeded_normal((M, K), 5), cuda_dev), False, bwgemm.MX_BLOCK32)
    qb, sfb = bwgemm.quantize_mxfp4(_t(o.seeded_normal((K, N), 6), cuda_dev), True, bwgemm.MX_BLOCK32)
    nbytes = M * N * 2
    whole, start = _guarded(nbytes, cuda_dev)
    C = _payload(whole, start, nbytes, torch.bfloat16, (M, N))
    bwgemm.gemm_mxfp4(qa, qb, sfa, sfb, K, C=C)
    _check(whole, start, nbytes)


@pytest.mark.parametrize("rows,cols", [(37, 48), (200, 328), (4096, 160), (130, 66)])
@pytest.mark.parametrize("transpose", [False, True])
def test_quantiser_writes_stay_inside_outputs(cuda_dev, rows, cols, transpose):
    import torch

    x = _t(o.seeded_normal((rows, cols), 7), cuda_dev)
    n = rows * cols
    w8, s8 = _guarded(n, cuda_dev)
    bwgemm.quantize_fp8(x, transpose, bwgemm.SCALE_AMAX,
                        dst=_payload(w8, s8, n, torch.uint8, (cols, rows) if transpose else (rows, cols)))
    _check(w8, s8, n)
    if (cols if not transpose else rows) % 2 == 0:
        w4, s4 = _guarded(n // 2, cuda_dev)
        bwgemm.quantize_fp4(x, transpose, bwgemm.SCALE_AMAX, bwgemm.FP4_PACKED,
                            dst=_payload(w4, s4, n // 2, torch.uint8,
                                         (cols, rows // 2) if transpose else (rows, cols // 2)))
        _check(w4, s4, n // 2)
    K = rows if transpose else cols
    outer = cols if transpose else rows
    if K % 32 == 0:
        nsf = bwgemm.sf_bytes(outer, K)
        wq, sq = _guarded(outer * K // 2, cuda_dev)
        wsf, ssf = _guarded(nsf, cuda_dev)
        bwgemm.quantize_mxfp4(x, transpose, bwgemm.MX_BLOCK32,
                              dst=_payload(wq, sq, outer * K // 2, torch.uint8, (outer, K // 2)),
                              sf=_payload(wsf, ssf, nsf, torch.uint8, (nsf,)))
        _check(wq, sq, outer * K // 2)
        _check(wsf, ssf, nsf)
