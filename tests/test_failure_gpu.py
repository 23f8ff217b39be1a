"""Failure detection without faulting the GPU: a kernel whose barrier is never signalled must
give up after its wait budget, report BW_ERR_TIMEOUT through the status word, and leave the
context usable for the next GEMM."""
import time

import numpy as np
import pytest

import bwgemm
import oracle as o

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda_dev):
    import torch

    L = bwgemm.lib()
    t0 = time.perf_counter()
    rc = L.bw_selftest_bounded_wait(20_000_000, torch.cuda.current_stream().cuda_stream)  # 20 ms
    dt = time.perf_counter() - t0
    assert rc == bwgemm.BW_ERR_TIMEOUT
    assert b"site 99" in L.bw_last_error_string()
    assert dt < 5.0
    assert bwgemm.device_status() == 0  # the word was read and cleared
    A = o.f16_to_f32(o.f32_to_f16(o.seeded_uniform((256, 256), 1)))
    C = bwgemm.gemm_f16(torch.from_numpy(A).to(cuda_dev).half(), torch.from_numpy(A).to(cuda_dev).half())
    torch.cuda.synchronize()
    assert np.abs(C.cpu().numpy() - o.gemm_f64(A, A)).max() <= o.f16_tolerance(256, 1, 1)


def test_selftest_rejects_bad_budget(cuda_dev):
    assert bwgemm.lib().bw_selftest_bounded_wait(0, None) == bwgemm.BW_ERR_INVALID
