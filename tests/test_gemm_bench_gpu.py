"""The reference-facing driver end to end: gemm_bench with the reference's command line and
inputs (glibc rand(), uniform[-0.5, 0.5]) must reproduce the reference's committed
max_abs_err column (results/bench.csv rows at 512^3, 1024^3 and 8192^3 of the reference repo) for our
tcgen05 rows, write the reference's CSV schema, and honour the kernel filter."""
import csv
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(REPO, "blackwell-tensorcore-kernels_b200", "gemm_bench")

# reference results/bench.csv: wmma/mma_* (fp16), mma_fp8, mma_fp4, mma_mxfp4
REF = {512: {"tc_f16": 0.00254, "tc_fp8": 0.283, "tc_fp4": 1.16, "tc_mxfp4": 1.16},
       1024: {"tc_f16": 0.00376, "tc_fp8": 0.439, "tc_fp4": 1.87, "tc_mxfp4": 1.87},
       8192: {"tc_f16": 0.0112, "tc_fp8": 1.4, "tc_fp4": 5.97, "tc_mxfp4": 5.97}}  # bench.csv:64,69-72


def _run(n, tmp_path, kernels):
    out = tmp_path / f"bench_{n}.csv"
    env = dict(os.environ, BW_INPUT_DIST="ref")
    r = subprocess.run([BIN, str(n), str(n), str(n), str(out), kernels], capture_output=True, text=True, env=env,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    with open(out) as f:
        return list(csv.DictReader(f)), r.stdout


@pytest.mark.parametrize("n", [512, 1024, 8192])
def test_reference_max_abs_err_column(tmp_path, n):
    rows, _ = _run(n, tmp_path, "tc_f16,tc_fp8,tc_fp4,tc_mxfp4,cublas_tc,cublaslt_fp8")
    got = {r["kernel"]: float(r["max_abs_err"]) for r in rows}
    for k, want in REF[n].items():
        assert abs(got[k] - want) <= 1.01e-2 * want, (k, got[k], want)
    # same math as the library rows on the same card
    assert abs(got["tc_f16"] - got["cublas_tc"]) <= 2e-5
    assert abs(got["tc_fp8"] - got["cublaslt_fp8"]) <= 1e-2 * got["tc_fp8"]


def test_csv_schema_and_filter(tmp_path):
    rows, stdout = _run(512, tmp_path, "tc_f16,tc_fp8_amax,tc_mxfp4_b32,tc_fp4_amax")
    assert [r["kernel"] for r in rows] == ["tc_f16", "tc_fp8_amax", "tc_fp4_amax", "tc_mxfp4_b32"]
    ref_cols = ["device", "sm", "M", "N", "K", "kernel", "ms", "tflops", "pct_of_cublas", "max_abs_err"]
    assert list(rows[0].keys())[:10] == ref_cols
    for r in rows:
        assert r["sm"] == "100" and float(r["tflops"]) > 0
        assert float(r["max_abs_err"]) < 2.0  # quantisation error of the scaled rows at 512^3


def test_appends_reference_shaped_rows_to_a_reference_csv(tmp_path):
    out = tmp_path / "old.csv"
    out.write_text("device,sm,M,N,K,kernel,ms,tflops,pct_of_cublas,max_abs_err\n")
    r = subprocess.run([BIN, "256", "256", "256", str(out), "tc_f16"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    lines = out.read_text().strip().splitlines()
    assert len(lines) == 2 and lines[1].count(",") == 9  # ten columns; the quoted device name holds no comma


def test_reference_rows_through_bw_ref_lib(tmp_path):
    """With BW_REF_LIB naming the reference's own launchers (built from its sources into
    oracle/_ref), the driver adds their rows beside ours; on B200 they reproduce the
    reference's own published max_abs_err at 1024^3 (mma_warptile/wmma 0.00376, mma_fp8 0.439),
    and without BW_REF_LIB there are no ref_* rows at all."""
    lib = os.path.join(REPO, "oracle", "_ref", "libref_kernels.so")
    if not os.path.exists(lib):
        pytest.fail(f"{lib} is missing: build it with oracle/build_ref.sh beside the reference checkout")
    out = tmp_path / "ref.csv"
    env = dict(os.environ, BW_INPUT_DIST="ref", BW_REF_LIB=lib)
    names = "tc_f16,ref_wmma,ref_mma_warptile,ref_mma_fp8"
    r = subprocess.run([BIN, "1024", "1024", "1024", str(out), names], capture_output=True, text=True, env=env,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    got = {row["kernel"]: float(row["max_abs_err"]) for row in csv.DictReader(open(out))}
    for k, want in {"ref_wmma": 0.00376, "ref_mma_warptile": 0.00376, "ref_mma_fp8": 0.439}.items():
        assert abs(got[k] - want) <= 1.01e-2 * want, (k, got[k], want)
    out2 = tmp_path / "noref.csv"
    env.pop("BW_REF_LIB")
    r = subprocess.run([BIN, "256", "256", "256", str(out2), names], capture_output=True, text=True, env=env,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    assert [row["kernel"] for row in csv.DictReader(open(out2))] == ["tc_f16"]
