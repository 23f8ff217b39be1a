"""Our device quantisers against the reference's OWN staging kernels, byte for byte.

The reference's q_fp8 / q_fp8_t / q_fp4 / q_fp4_t / q_mxfp4 / q_mxfp4_t
(src/gemm_mma_fp8.cu:37-80 of waynehacking8/blackwell-tensorcore-kernels) are compiled from its
sources for sm_100a into oracle/_ref/libref_kernels.so (oracle/build_ref.sh) and run here on
the same inputs as ours, with the reference's pre-scale of 8 for the FP4 forms:
  q_fp8(_t)    <-> bw_quantize_fp8(SCALE_NONE)                     (E4M3 satfinite, B -> Bt)
  q_fp4(_t)    <-> bw_quantize_fp4(SCALE_FIXED8, FP4_BYTE_SHL2)    (code << 2 byte container)
  q_mxfp4(_t)  <-> bw_quantize_mxfp4(MX_UNIT_FIXED8) codes          (two codes a byte, low nibble first)
Inputs: the golden edge-case tensor (ties, saturation, NaN/Inf, subnormals) and larger seeded
tensors at the reference's [-0.5, 0.5] range and at N(0, 1), including exact E2M1 midpoints.
"""
import ctypes
import os

import numpy as np
import pytest

import bwgemm

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(REPO, "oracle", "_ref", "libref_kernels.so")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_LIB):
        pytest.fail(f"{REF_LIB} is missing: build it with oracle/build_ref.sh beside the reference checkout")
    L = ctypes.CDLL(REF_LIB)
    L.ref_quant.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                            ctypes.c_float]
    L.ref_quant.restype = ctypes.c_int
    return L


def _inputs():
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "quant_golden.npz"))
    rng = np.random.default_rng(77)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32) / 8.0  # E2M1 ties after x 8
    tie = rng.choice(np.concatenate([mids, -mids]), size=(96, 256)).astype(np.float32)
    return {
        "golden_64x128": g["x"],
        "ref_range_1000x2048": (rng.random((1000, 2048), dtype=np.float32) - 0.5),
        "normal_512x4096": rng.standard_normal((512, 4096)).astype(np.float32),
        "ties_96x256": tie,
    }


def _run_ref(ref, name, x, out_shape, dev, scale=8.0):
    import torch

    src = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    out = torch.zeros(out_shape, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    rc = ref.ref_quant(name.encode(), src.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1], scale)
    torch.cuda.synchronize()  # the reference launches on the legacy default stream
    assert rc == 0, (name, rc)
    return out.cpu().numpy()


@pytest.mark.parametrize("case", list(_inputs().keys()))
@pytest.mark.parametrize("transpose", [False, True])
def test_fp8_matches_reference_q_fp8(cuda_dev, ref, case, transpose):
    import torch

    x = _inputs()[case]
    rows, cols = x.shape
    want = _run_ref(ref, "q_fp8_t" if transpose else "q_fp8", x, (cols, rows) if transpose else (rows, cols), cuda_dev)
    q, _ = bwgemm.quantize_fp8(torch.from_numpy(x).to(cuda_dev), transpose, bwgemm.SCALE_NONE)
    assert np.array_equal(q.cpu().numpy(), want)


@pytest.mark.parametrize("case", list(_inputs().keys()))
@pytest.mark.parametrize("transpose", [False, True])
def test_fp4_matches_reference_q_fp4(cuda_dev, ref, case, transpose):
    import torch

    x = _inputs()[case]
    rows, cols = x.shape
    want = _run_ref(ref, "q_fp4_t" if transpose else "q_fp4", x, (cols, rows) if transpose else (rows, cols), cuda_dev)
    q, _ = bwgemm.quantize_fp4(torch.from_numpy(x).to(cuda_dev), transpose, bwgemm.SCALE_FIXED8,
                               bwgemm.FP4_BYTE_SHL2)
    assert np.array_equal(q.cpu().numpy(), want)


@pytest.mark.parametrize("case", list(_inputs().keys()))
@pytest.mark.parametrize("transpose", [False, True])
def test_mxfp4_matches_reference_q_mxfp4(cuda_dev, ref, case, transpose):
    import torch

    x = _inputs()[case]
    rows, cols = x.shape
    K, outer = (rows, cols) if transpose else (cols, rows)
    if K % 32:
        pytest.skip("the block-scaled container needs K % 32 == 0")
    want = _run_ref(ref, "q_mxfp4_t" if transpose else "q_mxfp4", x, (outer, K // 2), cuda_dev)
    q, _ = bwgemm.quantize_mxfp4(torch.from_numpy(x).to(cuda_dev), transpose, bwgemm.MX_UNIT_FIXED8)
    assert np.array_equal(q.cpu().numpy(), want)
