"""GPU test of bw_quantize_fp8_noalloc, the quantiser entry point for callers that cannot
allocate device memory (stream callbacks, plugins inside a framework that has reserved the
device memory, serving loops with a no-allocation contract). It must give exactly what
bw_quantize_fp8 gives, call after call, although every call reuses the same fixed scratch
array inside the library. Collected last on purpose (file name), so a failure here cannot
stop the other GPU tests from running first.
"""
import numpy as np
import pytest

import bwgemm

pytestmark = pytest.mark.gpu


def _via_abi(fn, src, transpose, mode):
    import torch

    rows, cols = src.shape
    dst = torch.empty((cols, rows) if transpose else (rows, cols), dtype=torch.uint8, device=src.device)
    scale = torch.empty(1, dtype=torch.float32, device=src.device)
    rc = fn(src.data_ptr(), dst.data_ptr(), scale.data_ptr(), rows, cols, int(transpose), mode,
            torch.cuda.current_stream().cuda_stream)
    assert rc == bwgemm.BW_OK, bwgemm.lib().bw_last_error_string()
    return dst, scale


@pytest.mark.parametrize("transpose", [False, True])
@pytest.mark.parametrize("mode", [bwgemm.SCALE_AMAX, bwgemm.SCALE_NONE])
def test_noalloc_matches_allocating_entry_point_twice(cuda_dev, transpose, mode):
    import torch

    L = bwgemm.lib()
    g = torch.Generator(device=cuda_dev)
    g.manual_seed(7)
    # two calls in a row; the second input has a much smaller amax, so a stale maximum left in
    # the shared scratch by the first call would change its scale and codes
    first = torch.randn((1000, 1536), generator=g, device=cuda_dev) * 7.0
    second = torch.randn((777, 2304), generator=g, device=cuda_dev) * 0.01
    for src in (first, second):
        q_ref, s_ref = _via_abi(L.bw_quantize_fp8, src, transpose, mode)
        q_new, s_new = _via_abi(L.bw_quantize_fp8_noalloc, src, transpose, mode)
        torch.cuda.synchronize()
        assert torch.equal(q_new, q_ref)
        assert torch.equal(s_new, s_ref)


def test_noalloc_rejects_inputs_beyond_its_scratch(cuda_dev):
    import torch

    L = bwgemm.lib()
    src = torch.zeros(16, device=cuda_dev)
    dst = torch.zeros(16, dtype=torch.uint8, device=cuda_dev)
    # 16384 x 8193 elements is one block more than the fixed scratch can reduce; rejected
    # before any launch (the tiny buffers are never touched)
    rc = L.bw_quantize_fp8_noalloc(src.data_ptr(), dst.data_ptr(), None, 16384, 8193, 0, bwgemm.SCALE_AMAX,
                                   torch.cuda.current_stream().cuda_stream)
    assert rc == bwgemm.BW_ERR_INVALID
    assert b"scratch limit" in L.bw_last_error_string()
