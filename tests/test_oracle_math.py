"""Accuracy of the fp32 Exp/Tanh stand-ins the oracle and the kernels share.

Delphi's RTL Exp/Tanh are unavailable; the oracle and the CUDA kernels both use
g4_expf / g4_tanhf (identical IEEE operation sequences).  These tests bound
their error against libm in double precision, so the stand-in is as faithful
as a correctly-behaved RTL to within one ulp.
"""
import math

import numpy as np


def _ulps(got, ref):
    ref32 = np.float32(ref)
    if not np.isfinite(ref32):
        return 0.0 if got == ref32 else 1e9
    sp = abs(float(np.spacing(np.float32(abs(ref32)))))
    sp = max(sp, 1.4e-45)
    return abs(float(got) - ref) / sp


def test_g4_expf_within_one_ulp(oracle):
    lib = oracle.load()
    rng = np.random.default_rng(11)
    xs = np.concatenate([rng.uniform(-103.9, 88.7, 200000), rng.uniform(-2, 2, 100000),
                         np.array([0.0, -0.0, 1e-30, -1e-30, 88.7, -87.3, -100.0])]).astype(np.float32)
    worst = max(_ulps(lib.g4_expf(float(x)), math.exp(float(x))) for x in xs)
    assert worst <= 1.0, worst


def test_g4_expf_edges(oracle):
    lib = oracle.load()
    assert lib.g4_expf(float("inf")) == float("inf")
    assert lib.g4_expf(float("-inf")) == 0.0
    assert math.isnan(lib.g4_expf(float("nan")))
    assert lib.g4_expf(100.0) == float("inf")
    assert lib.g4_expf(-200.0) == 0.0
    assert lib.g4_expf(0.0) == 1.0


def test_g4_tanhf_within_one_ulp(oracle):
    lib = oracle.load()
    rng = np.random.default_rng(12)
    xs = np.concatenate([rng.uniform(-1, 1, 200000), rng.uniform(-12, 12, 100000),
                         rng.uniform(-1e-3, 1e-3, 20000),
                         np.array([0.0, 1.0, -1.0, 1.0000001, 9.0, 20.0, 1e-20])]).astype(np.float32)
    worst = max(_ulps(lib.g4_tanhf(float(x)), math.tanh(float(x))) for x in xs)
    assert worst <= 1.0, worst


def test_g4_tanhf_edges(oracle):
    lib = oracle.load()
    assert lib.g4_tanhf(float("inf")) == 1.0
    assert lib.g4_tanhf(float("-inf")) == -1.0
    assert math.isnan(lib.g4_tanhf(float("nan")))
    assert lib.g4_tanhf(0.0) == 0.0
    assert lib.g4_tanhf(50.0) == 1.0
    assert lib.g4_tanhf(-7.0) == -lib.g4_tanhf(7.0)


def test_rmsnorm_restatement(oracle):
    # CpuRmsNorm (src/Gemma4.Layers.pas:142-175) against an fp64 evaluation
    rng = np.random.default_rng(5)
    x = rng.standard_normal(2560).astype(np.float32) * 3
    w = rng.uniform(0.5, 1.5, 2560).astype(np.float32)
    got = oracle.rmsnorm(x, w, 1e-6)
    xd = x.astype(np.float64)
    want = xd / np.sqrt(np.mean(xd * xd) + 1e-6) * w
    assert np.max(np.abs(got - want) / np.abs(want)) < 1e-5


def test_lmhead_dequant_identities_exact():
    # The LM head turns a Q4_0 nibble n (0..15) and the block's fp16 scale s into
    # the fp16 weight (n - 8) * s rounded once, without an integer-to-float
    # conversion: the even nibbles of a word are masked in place as the fp16
    # value 1024 + n, the odd ones as 1024 + 16 n (both exact), then
    #   even: ((1024 + n) - 1032) * s
    #   odd:  fma(1024 + 16 n, 1/16, -72) * s
    # The subtraction and the fused multiply-add give n - 8 exactly, so the
    # product with s is the only rounding.  Checked for every nibble against a
    # sweep of scales (normal, subnormal, large, both signs).
    rng = np.random.default_rng(7)
    scales = np.concatenate([
        rng.standard_normal(20000).astype(np.float16),
        (rng.random(2000) * 0.02).astype(np.float16),                       # the C4 weight scales
        np.array([6.1e-5, 5.96e-8, -3e-6, 1e-7, 4094.0, -65504 / 16, 1.0, -1.0], dtype=np.float16),
    ])
    s32 = scales.astype(np.float32)
    for n in range(16):
        want = (np.float32(n - 8) * s32).astype(np.float16)                 # exact product, one rounding
        even = np.float16(1024 + n) - np.float16(1032)                      # exact in fp16
        odd = np.float16(np.float32(1024 + 16 * n) * np.float32(1 / 16) - np.float32(72))  # fma, exact
        assert float(even) == n - 8 and float(odd) == n - 8
        got_even = (np.float32(even) * s32).astype(np.float16)
        got_odd = (np.float32(odd) * s32).astype(np.float16)
        assert np.array_equal(got_even.view(np.uint16), want.view(np.uint16))
        assert np.array_equal(got_odd.view(np.uint16), want.view(np.uint16))
    # the masks: the bit patterns 0x6400 | n and 0x6400 | (n << 4) are those values
    for n in range(16):
        assert float(np.array([0x6400 | n], dtype=np.uint16).view(np.float16)[0]) == 1024 + n
        assert float(np.array([0x6400 | (n << 4)], dtype=np.uint16).view(np.float16)[0]) == 1024 + 16 * n
