"""The attention softmax's FMA-pipe exponential (``ex2_fma2`` in ``csrc/attention.cu``) on the CPU:
the polynomial coefficients are read from the kernel source and the same float32 steps (clamp,
1.5 * 2^23 shifter, Horner, exponent-field add) are evaluated over the argument range the
softmax produces (x <= 8 after the lazy rescale; masked keys give -inf).  Bound: relative error
<= 1e-4 against 2^x, far below the 2^-9 rounding of the bf16 P it feeds; 2^-inf and anything
below -125 give a value under 2^-125.  The GPU parity of the kernel itself is in
test_attention_gpu.py."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "fastworld_b200", "csrc",
                   "attention.cu")


def _coefficients():
    src = open(SRC).read()
    body = src[src.index("float2 ex2_fma2("):]
    body = body[:body.index("\n}\n")]
    vals = [float(v) for v in re.findall(r"make_float2\(([0-9.]+)f, \1f\)", body)]
    # Horner order in the source: c3 (first factor), c2, c1, c0 (shifter constants excluded)
    coef = [v for v in vals if v < 2.0]
    assert len(coef) == 4, coef
    return [np.float32(c) for c in coef]


def _ex2_fma(x):
    c3, c2, c1, c0 = _coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    sh = np.float32(12582912.0)
    t = (x + sh).astype(np.float32)
    nf = (t - sh).astype(np.float32)
    f = (x - nf).astype(np.float32)
    p = (c3 * f + c2).astype(np.float32)
    p = (p * f + c1).astype(np.float32)
    p = (p * f + c0).astype(np.float32)
    bits = (p.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << 23)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32)


def test_fma_exp2_relative_error():
    x = np.linspace(-124.0, 8.0, 2_000_001, dtype=np.float32)
    got = _ex2_fma(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    assert float(np.max(np.abs(got - ref) / ref)) <= 1e-4


def test_fma_exp2_masked_and_tiny_arguments():
    x = np.array([-np.inf, -1e30, -200.0, -125.5, -125.0], dtype=np.float32)
    got = _ex2_fma(x)
    assert np.all(np.isfinite(got)) and np.all(got >= 0) and np.all(got < 2.0 ** -124)
