"""CPU checks of the oracle against the reference's own known answers and element rules.

The reference has no test suite; its pins are the committed max_abs_err values in
results/bench.csv (rows 4,10-12 at 512^3 and 19,25-27 at 1024^3 of the reference repo), which
compare each kernel with cublasSgemm on glibc-rand() inputs. Reproducing them pins the
oracle's input generator, fp16/e4m3/e2m1 quantisers, FP4 byte container and MXFP4 packing.
"""
import json
import os
import subprocess

import numpy as np
import pytest

import oracle as o

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _ref_compat_errors(n):
    A, B = o.ref_fill_rand(n, n, n)
    R = o.gemm_f64(A, B)
    A16 = o.f16_to_f32(o.f32_to_f16(A))
    B16 = o.f16_to_f32(o.f32_to_f16(B))
    e16 = np.abs(o.gemm_f64(A16, B16) - R).max()
    qa, _ = o.quant_fp8(A, False, o.SCALE_NONE)
    qb, _ = o.quant_fp8(B, True, o.SCALE_NONE)
    e8 = np.abs(o.gemm_f64(o.dequant_fp8(qa), o.dequant_fp8(qb), b_trans=True) - R).max()
    qa, _ = o.quant_fp4(A, False, o.SCALE_FIXED8, o.FP4_BYTE_SHL2)
    qb, _ = o.quant_fp4(B, True, o.SCALE_FIXED8, o.FP4_BYTE_SHL2)
    e4 = np.abs(o.gemm_f64(o.dequant_fp4_byte(qa), o.dequant_fp4_byte(qb), b_trans=True) / 64 - R).max()
    qa, sa = o.quant_mxfp4(A, False, o.MX_UNIT_FIXED8)
    qb, sb = o.quant_mxfp4(B, True, o.MX_UNIT_FIXED8)
    em = np.abs(o.gemm_f64(o.dequant_mxfp4(qa, sa, n), o.dequant_mxfp4(qb, sb, n), b_trans=True) / 64 - R).max()
    return e16, e8, e4, em


# results/bench.csv of the reference: (fp16 wmma/mma_*, mma_fp8, mma_fp4, mma_mxfp4) max_abs_err
REF_MAX_ABS_ERR = {512: (0.00254, 0.283, 1.16, 1.16), 1024: (0.00376, 0.439, 1.87, 1.87)}


@pytest.mark.parametrize("n", [512, 1024])
def test_reference_max_abs_err_column(n):
    got = _ref_compat_errors(n)
    for g, want in zip(got, REF_MAX_ABS_ERR[n]):
        # 3 significant figures; the last digit may move by one because the reference's
        # check runs FP32 accumulation against cublasSgemm rather than FP64.
        assert abs(g - want) <= 1.01e-2 * want, (n, got, REF_MAX_ABS_ERR[n])


def test_glibc_rand_first_value():
    A, _ = o.ref_fill_rand(1, 1, 1)
    assert A[0, 0] == np.float32(1804289383 / np.float32(2147483647)) - np.float32(0.5)


def test_e2m1_rule_edges():
    # levels map to themselves, ties go to the smaller magnitude, > 6 saturates, NaN -> +0
    cases = {0.0: 0, 0.5: 1, 1.0: 2, 1.5: 3, 2.0: 4, 3.0: 5, 4.0: 6, 6.0: 7,
             0.25: 0, 0.75: 1, 1.25: 2, 1.75: 3, 2.5: 4, 3.5: 5, 5.0: 6, 7.0: 7, 100.0: 7,
             -0.75: 9, -6.5: 15, -0.0: 0, float("nan"): 0, float("inf"): 0, -float("inf"): 8,
             2.0 ** 30: 0, 1e-30: 0, -1e-30: 8}
    for v, want in cases.items():
        assert o.e2m1_code(v) == want, (v, o.e2m1_code(v), want)


def test_e4m3_edges():
    cases = {0.0: 0x00, 448.0: 0x7E, 1e9: 0x7E, -1e9: 0xFE, float("inf"): 0x7E, 464.0: 0x7E,
             1.0: 0x38, 2.0 ** -9: 0x01, 2.0 ** -10: 0x00, 1.5 * 2.0 ** -10: 0x01, float("nan"): 0x7F}
    for v, want in cases.items():
        assert o.e4m3_code(v) == want, (v, hex(o.e4m3_code(v)), hex(want))


def test_conversions_pinned_against_cuda_host_functions(tmp_path):
    """fp32->fp16 and fp32->e4m3 of the oracle equal CUDA's host conversions (strided sweep;
    the full 2^32 sweep is the `slow` test below)."""
    exe = _build_pin(tmp_path)
    r = subprocess.run([exe, "4099"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.slow
def test_conversions_pinned_exhaustive(tmp_path):
    exe = _build_pin(tmp_path)
    r = subprocess.run([exe, "1"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def _build_pin(tmp_path):
    here = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle")
    obj = str(tmp_path / "bo.o")
    exe = str(tmp_path / "pin")
    subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-c", os.path.join(here, "bw_oracle.c"), "-o", obj],
                   check=True)
    subprocess.run(["g++", "-O2", "-std=c++17", "-I/usr/local/cuda/include", os.path.join(here, "pin_conversions.cpp"),
                    obj, "-o", exe, "-lm", "-lpthread"], check=True)
    return exe


def _build_e2m1_check(tmp_path):
    here = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle")
    exe = str(tmp_path / "e2m1")
    subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", os.path.join(here, "check_e2m1_fast.c"),
                    os.path.join(here, "bw_oracle.c"), "-o", exe, "-lm", "-lpthread"], check=True)
    return exe


def test_fast_e2m1_encoder_matches_rule(tmp_path):
    """The quantisers' table-driven E2M1 encoder equals the reference rule (strided sweep of
    all bit patterns, every NaN/Inf/subnormal class included; the full sweep is `slow`)."""
    r = subprocess.run([_build_e2m1_check(tmp_path), "97"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.slow
def test_fast_e2m1_encoder_matches_rule_exhaustive(tmp_path):
    r = subprocess.run([_build_e2m1_check(tmp_path), "1"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_mx_scale_rule():
    # block amax in [2^(e+2), 2^(e+3)) -> byte e + 127; all-zero block -> byte 0
    x = np.zeros((1, 128), np.float32)
    x[0, 0:32] = 1.0          # amax 1 -> e = -2 -> 125
    x[0, 32:64] = 7.99        # amax 7.99 -> e = 0 -> 127; 7.99 saturates to 6
    x[0, 64:96] = 0.0         # zero block -> 0
    x[0, 96:128] = -96.0      # amax 96 -> floor(log2) = 6 -> e = 4 -> 131
    q, sf = o.quant_mxfp4(x, False, o.MX_BLOCK32)
    got = [int(sf[o.sf_offset(0, j, 128)]) for j in range(4)]
    assert got == [125, 127, 0, 131]
    deq = o.dequant_mxfp4(q, sf, 128)
    assert deq[0, 0] == 1.0 and deq[0, 40] == 6.0 and deq[0, 70] == 0.0 and deq[0, 100] == -96.0


def test_sf_layout_matches_tiled_formula():
    K, outer = 512, 300
    assert o.sf_bytes(outer, K) == 3 * 4 * 512
    seen = set()
    for r in range(outer):
        for j in range(K // 32):
            off = o.sf_offset(r, j, K)
            assert off not in seen
            seen.add(off)
            rr = r % 128
            assert off % 512 == (rr % 32) * 16 + (rr // 32) * 4 + j % 4


def test_golden_fixtures_match_oracle():
    """Committed fixtures (tests/golden/make_golden.py) still match the oracle."""
    path = os.path.join(GOLDEN, "quant_golden.npz")
    if not os.path.exists(path):
        pytest.fail("tests/golden/quant_golden.npz missing: run tests/golden/make_golden.py")
    g = np.load(path)
    x = g["x"]
    q, _ = o.quant_fp8(x, False, o.SCALE_NONE)
    assert np.array_equal(q, g["fp8"])
    q, _ = o.quant_fp4(x, False, o.SCALE_FIXED8, o.FP4_BYTE_SHL2)
    assert np.array_equal(q, g["fp4_byte"])
    q, sf = o.quant_mxfp4(x, False, o.MX_UNIT_FIXED8)
    assert np.array_equal(q, g["mxfp4_ref"])
    q, sf = o.quant_mxfp4(x, False, o.MX_BLOCK32)
    assert np.array_equal(q, g["mxfp4_q"]) and np.array_equal(sf, g["mxfp4_sf"])
    assert np.array_equal(o.f32_to_f16(x), g["f16"])
    meta = json.loads(str(g["meta"]))
    assert meta["rows"] == x.shape[0]
