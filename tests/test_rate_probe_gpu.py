"""tcgen05 issue-rate probe (the B200 analogue of the reference's src/mma_rate_probe.cu:63-114,
whose output the reference commits as results/mma_rate_probe.csv): one CTA per SM issues
back-to-back MMAs from resident shared-memory operands, and the clock64-timed rate per SM must
sit within 10% of the tensor core's per-clock issue rate for each kind. These per-clock
figures are the denominators of the FLOP/SM/clk efficiencies the kernels report."""
import csv
import os
import statistics
import subprocess

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(REPO, "blackwell-tensorcore-kernels_b200", "tc_rate_probe")

# dense FLOP per SM per clock: kind::f16 M128 N256 K16 in 128 clk, f8f6f4 twice, mxf4 four times
EXPECTED = {"f16_m128n256k16": 8192.0, "e4m3_m128n256k32": 16384.0, "mxf4_m128n256k64": 32768.0,
            "f16_pair_m256n256k16": 8192.0, "mxf4_pair_m256n256k64": 32768.0}


def test_rate_probe_per_clock_rates(tmp_path):
    out = tmp_path / "probe.csv"
    r = subprocess.run([BIN, "2048", "3", str(out)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    rows = list(csv.DictReader(open(out)))
    assert set(EXPECTED) <= {row["variant"] for row in rows}
    for name, want in EXPECTED.items():
        got = statistics.median(float(row["flop_per_sm_clk"]) for row in rows if row["variant"] == name)
        assert abs(got - want) <= 0.10 * want, (name, got, want)
        mhz = statistics.median(float(row["sm_mhz_effective"]) for row in rows if row["variant"] == name)
        assert 500.0 < mhz < 2100.0, (name, mhz)
