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
                 "bw_unshard_columns", "bw_gemm_sharded"]:
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


def test_sharded_argument_validation_without_gpu():
    L = bwgemm.lib()
    S = bwgemm.Shard
    buf = ctypes.create_string_buffer(256)
    p = (ctypes.addressof(buf) + 15) & ~15

    def call(dtype, out, parts, M, N, K, gather):
        arr = (S * max(1, len(parts)))(*parts)
        return L.bw_gemm_sharded(dtype, out, ctypes.cast(arr, ctypes.c_void_p), len(parts), M, N, K, gather)

    ok = S(0, p, p, None, None, None, None, p, None, None)
    assert call(7, 0, [ok], 8, 8, 8, 0) == bwgemm.BW_ERR_INVALID                      # dtype
    assert call(bwgemm.DTYPE_F16, bwgemm.OUT_BF16, [ok], 8, 8, 8, 0) == bwgemm.BW_ERR_INVALID  # FP16 writes FP32
    assert L.bw_gemm_sharded(0, 0, None, 1, 8, 8, 8, 0) == bwgemm.BW_ERR_INVALID    # no shards
    assert call(0, 0, [], 8, 8, 8, 0) == bwgemm.BW_ERR_INVALID                      # ngpu = 0
    two = [S(0, p, p, None, None, None, None, p, None, None), S(1, p, p, None, None, None, None, p, None, None)]
    assert call(0, 0, two, 8, 9, 8, 0) == bwgemm.BW_ERR_INVALID                     # N % ngpu
    assert b"divisible" in L.bw_last_error_string()
    dup = [S(0, p, p, None, None, None, None, p, None, None)] * 2
    assert call(0, 0, dup, 8, 8, 8, 0) == bwgemm.BW_ERR_INVALID                     # same device twice
    assert call(0, 0, two, 8, 8, 8, 1) == bwgemm.BW_ERR_INVALID                     # gather, no C_gathered
    assert call(bwgemm.DTYPE_MXFP4, 1, two, 8, 8, 64, 0) == bwgemm.BW_ERR_INVALID   # MXFP4 without sfA/sfB
    assert b"sfA" in L.bw_last_error_string()
    nul = [S(0, None, p, None, None, None, None, p, None, None)]
    assert call(0, 0, nul, 8, 8, 8, 0) == bwgemm.BW_ERR_INVALID                     # A null


def test_allgather_and_ipc_argument_validation_without_gpu():
    L = bwgemm.lib()
    buf = ctypes.create_string_buffer(256)
    p = (ctypes.addressof(buf) + 31) & ~31
    peers = (ctypes.c_void_p * 2)(p, p)
    assert L.bw_gemm_f16_allgather(p, p, p, peers, 0, 0, 8, 16, 8, None) == bwgemm.BW_ERR_INVALID  # world 0
    assert L.bw_gemm_f16_allgather(p, p, p, peers, 2, 2, 8, 16, 8, None) == bwgemm.BW_ERR_INVALID  # rank >= world
    assert L.bw_gemm_f16_allgather(p, p, p, peers, 2, 0, 8, 15, 8, None) == bwgemm.BW_ERR_INVALID  # N_total % world
    assert L.bw_gemm_f16_allgather(p, p, p, None, 2, 0, 8, 16, 8, None) == bwgemm.BW_ERR_INVALID   # no peers
    assert L.bw_gemm_fp8_allgather(p, p, None, None, p, 1, peers, 9, 0, 8, 16, 16, None) == bwgemm.BW_ERR_INVALID
    assert L.bw_ipc_malloc(0, None, None) == bwgemm.BW_ERR_INVALID
    assert L.bw_ipc_open(None, None) == bwgemm.BW_ERR_INVALID
    assert L.bw_ipc_free(None) == bwgemm.BW_OK and L.bw_ipc_close(None) == bwgemm.BW_OK
