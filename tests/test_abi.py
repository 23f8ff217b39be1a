"""CPU checks of the C ABI: the in-tree library loads, exports every entry point that
include/bwgemm.h declares, and rejects bad arguments before touching the GPU."""
import ctypes
import subprocess

import pytest

import bwgemm


def test_header_declares_the_expected_surface():
    names = set(bwgemm.declared_functions())
    for must in ["bw_init", "bw_gemm_f16", "bw_gemm_f16_bt", "bw_gemm_fp8", "bw_gemm_mxfp4", "bw_gemm_fp4",
                 "bw_quantize_f16", "bw_quantize_fp8", "bw_quantize_fp4", "bw_quantize_mxfp4",
                 "bw_last_error_string", "bw_device_status", "bw_sf_bytes", "bw_sf_offset",
                 "bw_unshard_columns"]:
        assert must in names, must


def test_library_exports_every_declared_symbol():
    L = bwgemm.lib()
    missing = [n for n in bwgemm.declared_functions() if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", bwgemm.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert set(bwgemm.declared_functions()) <= exported


def test_argument_validation_without_gpu():
    L = bwgemm.lib()
    assert L.bw_gemm_f16(None, None, None, -1, 8, 8, None) == bwgemm.BW_ERR_INVALID
    assert b"negative" in L.bw_last_error_string()
    assert L.bw_gemm_f16(None, None, None, 0, 8, 8, None) == bwgemm.BW_OK  # empty problem
    assert L.bw_gemm_fp8(None, None, None, None, None, 0, 4, 4, 4, None) == bwgemm.BW_ERR_INVALID  # C null
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    p16 = (p + 15) & ~15
    assert L.bw_gemm_f16(p16 + 1, p16, p16, 8, 8, 8, None) == bwgemm.BW_ERR_INVALID  # misaligned
    assert L.bw_quantize_mxfp4(None, None, None, 4, 48, 0, 1, None) == bwgemm.BW_ERR_INVALID  # K % 32
    assert L.bw_unshard_columns(None, None, 4, 10, 3, None) == bwgemm.BW_ERR_INVALID


def test_sf_layout_functions_match_oracle():
    import oracle as o

    for outer, K in [(1, 32), (128, 128), (300, 512), (257, 96)]:
        assert bwgemm.sf_bytes(outer, K) == o.sf_bytes(outer, K)
        for r in range(0, outer, 37):
            for j in range(K // 32):
                assert bwgemm.lib().bw_sf_offset(r, j, K) == o.sf_offset(r, j, K)
