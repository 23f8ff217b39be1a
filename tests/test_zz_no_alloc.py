"""GPU test of bw_quantize_fp8_noalloc, the quantiser entry point for callers that cannot
allocate device memory (plugins inside a framework that has reserved the device memory,
serving loops with a no-allocation contract). It must give exactly what
bw_quantize_fp8 gives, call after call, although every call reuses the same fixed scratch
array inside the library. Collected last on purpose (file name), so a failure here cannot
stop the other GPU tests from running first.
"""
import os
import subprocess
import sys

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
@pytest.mark.parametrize("mode", [bwgemm.SCALE_AMAX, bwgemm.SCALE_NONE, bwgemm.SCALE_FIXED8])
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


_FRESH = r"""
import ctypes, sys
import torch
sys.path.insert(0, sys.argv[1])
import bwgemm
L = bwgemm.lib()  # loads the library; bwgemm.init() is deliberately not called
torch.cuda.set_device(0)
src = torch.randn((513, 1024), device="cuda") * 3.0
dst = torch.empty((513, 1024), dtype=torch.uint8, device="cuda")
scale = torch.empty(1, dtype=torch.float32, device="cuda")
assert L.bw_device_state_ready(0) == 0
s = torch.cuda.current_stream().cuda_stream
for _ in range(2):
    rc = L.bw_quantize_fp8_noalloc(src.data_ptr(), dst.data_ptr(), scale.data_ptr(), 513, 1024, 0,
                                   bwgemm.SCALE_AMAX, s)
    assert rc == 0, L.bw_last_error_string()
torch.cuda.synchronize()
# the first library call of the process was the no-alloc one: the library state with its
# cudaMalloc'd workspace must still not exist
assert L.bw_device_state_ready(0) == 0, "library workspace was created"
q_ref, s_ref = bwgemm.quantize_fp8(src, False, bwgemm.SCALE_AMAX)  # sets the state up now
torch.cuda.synchronize()
assert L.bw_device_state_ready(0) == 1
assert torch.equal(dst, q_ref) and torch.equal(scale, s_ref)
print("fresh-process ok")
"""


def test_noalloc_as_first_call_of_a_fresh_process_creates_no_workspace(cuda_dev):
    pkg = os.path.dirname(bwgemm.__file__)
    r = subprocess.run([sys.executable, "-c", _FRESH, pkg], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "fresh-process ok" in r.stdout, r.stdout + r.stderr


def test_noalloc_tall_transposed_input(cuda_dev):
    """More row groups than one launch's grid.y holds (65535 x 128 rows): the transposing
    kernel walks the rest in a loop, in both entry points."""
    import torch

    L = bwgemm.lib()
    g = torch.Generator(device=cuda_dev)
    g.manual_seed(11)
    src = torch.randn((65535 * 128 + 272, 8), generator=g, device=cuda_dev)
    q_ref, s_ref = _via_abi(L.bw_quantize_fp8, src, True, bwgemm.SCALE_AMAX)
    q_new, s_new = _via_abi(L.bw_quantize_fp8_noalloc, src, True, bwgemm.SCALE_AMAX)
    torch.cuda.synchronize()
    assert torch.equal(q_new, q_ref) and torch.equal(s_new, s_ref)
    # the whole result against the CPU oracle (its rows past 65535 x 128 come from the loop)
    import oracle as o

    qr, sr = o.quant_fp8(src.cpu().numpy(), True, o.SCALE_AMAX)
    assert (q_ref.cpu().numpy() == qr).all() and float(s_ref.item()) == sr
