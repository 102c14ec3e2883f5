"""Error bound of exp2_fma (llminfer_b200/csrc/common.cuh), the FMA-pipe
2^x the tensor-core prefill uses for part of its softmax exponentials.

The device routine is emulated here step for step in IEEE float32 (the same
adds, fmas, integer shift and add), with the coefficients read from the CUDA
source so the two cannot drift apart, and compared with exact 2^x over the
range the softmax uses (score minus running max in [-125, 8]).  The bar is
the fp16 rounding the probabilities get next: 2^-11 relative.
"""
import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parent.parent / "llminfer_b200" / "csrc" / "common.cuh"


def coefficients():
    body = SRC.read_text().split("float exp2_fma(float x)")[1].split("}")[0]
    line = [l for l in body.splitlines() if "const float p" in l][0]
    return [np.float32(v) for v in re.findall(r"(-?\d+\.\d+)f", line)]  # c3, c2, c1, c0


def emulate(x):
    c3, c2, c1, c0 = coefficients()
    x = np.minimum(np.maximum(x, np.float32(-125)), np.float32(126)).astype(np.float32)
    shifter = np.float32(12582912.0)
    t = (x + shifter).astype(np.float32)
    f = (x - (t - shifter).astype(np.float32)).astype(np.float32)

    def fma(a, b, c):  # single rounding, as the device FFMA
        return (a.astype(np.float64) * b + c).astype(np.float32)

    p = fma(fma(fma(np.full_like(f, c3), f, c2), f, c1), f, c0)
    bits = (p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23))
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def test_exp2_fma_relative_error_below_fp16_rounding():
    x = np.concatenate([np.linspace(-125, 8, 1_000_001), -np.logspace(-9, 2, 20_000),
                        np.arange(-125, 9)]).astype(np.float32)
    got = emulate(x).astype(np.float64)
    rel = np.abs(got / np.exp2(x.astype(np.float64)) - 1.0)
    assert rel.max() < 1e-4 < 2.0 ** -11


def test_exp2_fma_is_monotone_enough_for_softmax():
    x = np.linspace(-20, 8, 200_001).astype(np.float32)
    y = emulate(x).astype(np.float64)
    # Never decreases by more than its error bound between neighbours.
    assert np.all(np.diff(y) >= -2e-4 * y[1:])
