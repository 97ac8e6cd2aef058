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
