"""Writes tests/golden/quant_golden.npz: quantiser outputs of the oracle on a fixed input that
covers the element-rule edges (E2M1 ties, saturation, NaN/Inf, subnormals, fp8 overflow).
The GPU tests compare the device quantisers with these bytes, so the fixture pins both.

    python tests/golden/make_golden.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as o  # noqa: E402


def make_input(rows=64, cols=128):
    rng = np.random.default_rng(20261201)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    x[0, :32] = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, 0.5, 1.0, 6.0, -0.75, -6.5, 0.0, -0.0, 100.0,
                 np.nan, np.inf, -np.inf, 1e-30, -1e-30, 2.0 ** 30, 448.0, 464.0, 1e9, -1e9, 2.0 ** -10,
                 1.5 * 2.0 ** -10, 65520.0, 6e-8, 3e-8, -3.0]
    x[1] *= 1e-6        # tiny block (subnormal-ish scales)
    x[2] *= 1e4         # large block
    x[3, :32] = 0.0     # all-zero MX block
    x[4] = x[4] / 8.0   # reference range ([-0.5, 0.5]-like) for the x8 paths
    return x


def main():
    x = make_input()
    fp8, _ = o.quant_fp8(x, False, o.SCALE_NONE)
    fp4b, _ = o.quant_fp4(x, False, o.SCALE_FIXED8, o.FP4_BYTE_SHL2)
    mxr, _ = o.quant_mxfp4(x, False, o.MX_UNIT_FIXED8)
    mxq, mxsf = o.quant_mxfp4(x, False, o.MX_BLOCK32)
    f16 = o.f32_to_f16(x)
    meta = json.dumps({"rows": x.shape[0], "cols": x.shape[1], "seed": 20261201,
                       "generator": "tests/golden/make_golden.py"})
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), x=x, fp8=fp8, fp4_byte=fp4b, mxfp4_ref=mxr,
                        mxfp4_q=mxq, mxfp4_sf=mxsf, f16=f16, meta=np.array(meta))
    print("wrote quant_golden.npz")


if __name__ == "__main__":
    main()
