"""The oracle's restatement of the reference's GPU LM head (Q8_1 activations,
shaders/src/gemma4_quantize_q8.comp; DP4A matvec, shaders/src/gemma4_matvec_q4q8.comp),
checked on the CPU against hand-derived values and an independent numpy
statement of the same formulas."""
import numpy as np

import synth


def _f16(bits):
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def test_quantize_known_answers(oracle):
    # amax 127 -> d = 1, id = 1: q = round(v), halves away from zero
    v = np.zeros(32, np.float32)
    v[:8] = [127.0, -127.0, 0.5, -0.5, 1.5, 2.5, -2.49, 3.7]
    qs, ds = oracle.quantize_q8_1(v)
    assert list(qs[:8]) == [127, -127, 1, -1, 2, 3, -2, 4]
    assert (qs[8:] == 0).all()
    assert _f16(ds[0, 0]) == 1.0
    assert _f16(ds[0, 1]) == float(qs.astype(np.int32).sum())
    # an all-zero block: d = 0, id = 0, q = 0
    qs, ds = oracle.quantize_q8_1(np.zeros(32, np.float32))
    assert (qs == 0).all() and (ds == 0).all()


def test_quantize_matches_numpy_statement(oracle):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(2560) * rng.uniform(0.01, 5, 2560)).astype(np.float32)
    qs, ds = oracle.quantize_q8_1(x)
    xb = x.reshape(-1, 32)
    amax = np.abs(xb).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    t = (xb * idv[:, None]).astype(np.float32)
    q = np.clip(np.sign(t) * np.floor(np.abs(t) + 0.5), -127, 127).astype(np.int8)
    np.testing.assert_array_equal(qs.reshape(-1, 32), q)
    # fp16 packing rounds to nearest even (numpy's float16 conversion does the same)
    np.testing.assert_array_equal(ds[:, 0], d.astype(np.float16).view(np.uint16))
    s = (d * q.astype(np.int32).sum(axis=1).astype(np.float32)).astype(np.float32)
    np.testing.assert_array_equal(ds[:, 1], s.astype(np.float16).view(np.uint16))


def test_matvec_q4q8_matches_numpy_statement(oracle):
    rows, H = 96, 512
    h, blocks = synth.c4_inputs(1, H, rows, seed=11)
    x = h[0]
    got = oracle.matvec_q4q8(blocks, x, rows, H, nthreads=3)
    qs, ds = oracle.quantize_q8_1(x)
    b = blocks.reshape(rows, H // 32, 18)
    nib = np.empty((rows, H // 32, 32), np.int32)
    nib[:, :, 0::2] = b[:, :, 2:] & 0x0F
    nib[:, :, 1::2] = b[:, :, 2:] >> 4
    idot = (nib * qs.reshape(1, -1, 32).astype(np.int32)).sum(axis=2)
    d4 = (b[:, :, 0].astype(np.uint16) | (b[:, :, 1].astype(np.uint16) << 8)).view(np.float16).astype(np.float64)
    d8 = _f16(ds[:, 0]).astype(np.float64)
    s8 = _f16(ds[:, 1]).astype(np.float64)
    want = (d4 * (d8[None, :] * idot - 8.0 * s8[None, :])).sum(axis=1)
    scale = (np.abs(d4) * (d8[None, :] * np.abs(idot) + 8 * np.abs(s8[None, :]))).sum(axis=1)
    assert (np.abs(got - want) <= 1e-6 * scale + 1e-30).all()


def test_matvec_paths_agree_within_quantisation(oracle):
    # the fp32 CPU path and the Q8_1 GPU path of the reference compute the same
    # logits up to the int8 rounding of the activations (|dq| <= d/2 per value)
    rows, H = 64, 2560
    h, blocks = synth.c4_inputs(1, H, rows, seed=12)
    x = h[0]
    y32 = oracle.matvec_q4(blocks, x, rows, H)
    y32mt = oracle.matvec_q4_mt(blocks, x, rows, H, nthreads=4)
    np.testing.assert_array_equal(y32, y32mt)
    y8 = oracle.matvec_q4q8(blocks, x, rows, H, nthreads=2)
    b = blocks.reshape(rows, H // 32, 18)
    d4 = (b[:, :, 0].astype(np.uint16) | (b[:, :, 1].astype(np.uint16) << 8)).view(np.float16).astype(np.float64)
    amax = np.abs(x.reshape(-1, 32)).max(axis=1) / 127.0
    # plus the fp16 rounding of d and s (2^-11 relative): a loose 1.25 factor
    bound = (np.abs(d4) * 8.0 * 32 * (amax[None, :] / 2)).sum(axis=1) * 1.25 + 1e-4
    assert (np.abs(y8.astype(np.float64) - y32) <= bound).all()
