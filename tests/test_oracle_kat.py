"""Known-answer tests of the CPU oracle, derived by hand from the reference source.

The reference ships no sampler tests or vectors, so these pin the oracle's
semantics directly against what src/Gemma4.Model.pas:2615-2827,
src/Gemma4.Layers.pas:300-316, src/Gemma4.Tensors.pas:546-674 and
src/Gemma4.Types.pas:417-500 compute, case by case.
"""
import math

import numpy as np
import pytest

F32, F64, LIBM = 0, 1, 2


def P(o, T=1.0, K=64, top_p=0.95):
    return o.params(T, K, top_p)


def test_index_order_draw_full_path(oracle):
    # 4 equal logits, no softcap, full path (K=0): p = 0.25 each; cumsum in id order
    x = np.zeros(4, np.float32)
    for u, want in [(0.0, 0), (0.1, 0), (0.26, 1), (0.6, 2), (0.99, 3)]:
        tok, tr, _, _ = oracle.sample(x, P(oracle, 1.0, 0, 1.0), 0.0, u, F32)
        assert tok == want, (u, tok)
        assert tr["path"] == oracle.PATH_FULL


def test_draw_is_not_a_sort(oracle):
    # the largest probability is NOT visited first: ids are scanned in ascending order
    x = np.array([0.0, 5.0, 0.0], np.float32)
    tok, tr, _, _ = oracle.sample(x, P(oracle, 1.0, 0, 1.0), 0.0, 0.001, F32)
    assert tok == 0  # id 0 reaches a tiny threshold first although id 1 dominates


def test_threshold_rounds_to_single(oracle):
    x = np.zeros(8, np.float32)
    tok, tr, _, _ = oracle.sample(x, P(oracle, 1.0, 0, 0.95), 0.0, 0.3, F32)
    assert tr["thr"] == np.float32(0.3 * np.float64(np.float32(0.95)))


def test_fallback_to_argmax_when_threshold_unreached(oracle):
    # top_p > 1: u * P can exceed the final cumsum (~1) -> argmax is kept
    x = np.array([0.0, 1.0, 3.0, 2.0], np.float32)
    tok, tr, _, _ = oracle.sample(x, P(oracle, 1.0, 0, 2.0), 0.0, 0.9, F32)
    assert tok == 2 and tr["fallback"] == 1
    tok, tr, _, _ = oracle.sample(x, P(oracle, 1.0, 3, 2.0), 0.0, 0.9, F32)
    assert tok == 2 and tr["fallback"] == 1 and tr["path"] == oracle.PATH_TOPK


def test_greedy_when_temperature_not_positive(oracle):
    x = np.array([0.5, 4.0, 4.0, -1.0], np.float32)
    for T in (0.0, -1.0):
        for K in (0, 2, 3):
            tok, tr, _, _ = oracle.sample(x, P(oracle, T, K, 0.9), 30.0, 0.999, F32)
            assert tok == 1 and tr["drawn"] == 0  # first maximum wins


def _topk_probs_by_hand(lib, vals, inv_t):
    v = [np.float32(a) for a in vals]
    if inv_t is not None:
        v = [np.float32(a * np.float32(inv_t)) for a in v]
    m = max(v)
    e = [np.float32(lib.g4_expf(np.float32(a - m))) for a in v]
    s = np.float32(0)
    for a in e:
        s = np.float32(s + a)
    return np.array([np.float32(a / s) for a in e], np.float32)


def test_temperature_scaling_rule(oracle):
    # T > 0 and T != 1: multiply by fl32(1/T); T == 1: no multiply at all
    lib = oracle.load()
    x = np.array([0.7, -1.3, 2.1, 0.2], np.float32)
    for T, inv in [(1.0, None), (0.5, 2.0), (3.0, np.float32(1.0) / np.float32(3.0))]:
        _, _, ids, pr = oracle.sample(x, P(oracle, T, 3, 1.0), 0.0, 0.5, F32, want_probs=True)
        assert list(ids) == [0, 2, 3]
        assert np.array_equal(pr, _topk_probs_by_hand(lib, x[[0, 2, 3]], inv)), T


def test_dispatch_topk_bounds(oracle):
    x = np.arange(10, dtype=np.float32)
    for K, path in [(0, 1), (-5, 1), (10, 1), (11, 1), (9, 0), (1, 0)]:
        _, tr, _, _ = oracle.sample(x, P(oracle, 1.0, K, 0.9), 30.0, 0.5, F32)
        assert tr["path"] == path, K


def test_topk_set_and_order(oracle):
    x = np.array([3.0, -1.0, 7.0, 7.0, 0.5, 9.0, 2.0], np.float32)
    ids = oracle.topk(x, 3, oracle.TIE_LOWER)
    assert list(ids) == [2, 3, 5]  # ascending ids, ties at 7 both inside
    ids = oracle.topk(x, 2, oracle.TIE_LOWER)
    assert list(ids) == [2, 5]  # tie at the K-th place: lower id wins


def test_heap_tie_differs_from_lower_index(oracle):
    # example worked through DoSelectTopKIndices by hand
    x = np.array([0, 0, 1, 2, 2, 1, 0], np.float32)
    assert list(oracle.topk(x, 5, oracle.TIE_HEAP)) == [1, 2, 3, 4, 5]
    assert list(oracle.topk(x, 5, oracle.TIE_LOWER)) == [0, 2, 3, 4, 5]


def test_topk_excludes_minus_1e30_and_below(oracle):
    x = np.array([-1e30, -np.inf, 1.0, -2e30, 0.0], np.float32)
    ids = oracle.topk(x, 4, oracle.TIE_HEAP)
    assert list(ids) == [2, 4]
    assert list(oracle.topk(x, 4, oracle.TIE_LOWER)) == [2, 4]


def test_empty_topk_row_returns_minus_one(oracle):
    x = np.full(6, -np.inf, np.float32)
    tok, tr, _, _ = oracle.sample(x, P(oracle, 1.0, 3, 0.9), 30.0, 0.5, F32)
    assert tok == -1 and tr["count"] == 0


def test_nan_maps_to_minus_inf(oracle):
    x = np.array([np.nan, 1.0, 2.0, np.nan], np.float32)
    y = np.array([-np.inf, 1.0, 2.0, -np.inf], np.float32)
    for K in (0, 2):
        a = oracle.sample(x, P(oracle, 1.0, K, 0.9), 30.0, 0.3, F32)[0]
        b = oracle.sample(y, P(oracle, 1.0, K, 0.9), 30.0, 0.3, F32)[0]
        assert a == b


def test_two_softcap_spellings(oracle):
    # top-K path: cap * tanh(v / cap); full path: tanh(v * (1/cap)) * cap
    lib = oracle.load()
    v = np.float32(17.3)
    cap = np.float32(30.0)
    a = np.float32(cap * np.float32(lib.g4_tanhf(np.float32(v / cap))))
    inv = np.float32(np.float32(1.0) / cap)
    b = np.float32(np.float32(lib.g4_tanhf(np.float32(v * inv))) * cap)
    assert abs(float(a) - 30 * math.tanh(17.3 / 30)) < 4e-6
    assert abs(float(b) - 30 * math.tanh(17.3 / 30)) < 4e-6
    # the K survivors are capped with the first form
    x = np.array([v, 0.0, -5.0], np.float32)
    _, _, ids, pr = oracle.sample(x, P(oracle, 1.0, 2, 1.0), 30.0, 0.5, F32, want_probs=True)
    e0 = np.float32(lib.g4_expf(np.float32(0.0)))
    e1 = np.float32(lib.g4_expf(np.float32(np.float32(0.0) - a)))
    s = np.float32(e0 + e1)
    assert list(ids) == [0, 1]
    assert pr[0] == np.float32(e0 / s) and pr[1] == np.float32(e1 / s)


def test_full_path_normalises_by_reciprocal(oracle):
    # CpuSoftmaxF32 multiplies by fl32(1/sum); the top-K path divides
    lib = oracle.load()
    x = np.array([0.3, 1.7, -0.4], np.float32)
    _, tr, _, pr = oracle.sample(x, P(oracle, 1.0, 0, 1.0), 0.0, 0.5, F32, want_probs=True)
    m = np.float32(1.7)
    e = np.array([lib.g4_expf(np.float32(v - m)) for v in x], np.float32)
    s = np.float32(0)
    for v in e:
        s = np.float32(s + v)
    inv = np.float32(np.float32(1.0) / s)
    assert np.array_equal(pr, (e * inv).astype(np.float32))


def test_bf16_widen_and_truncate(oracle):
    lib = oracle.load()
    assert lib.ref_bf16_to_f32(0x3F80) == 1.0
    assert lib.ref_bf16_to_f32(0xC040) == -3.0
    assert lib.ref_f32_to_bf16_trunc(np.float32(1.0078125 + 0.00390625)) == 0x3F81  # truncates


def test_f16_decode_and_encode(oracle):
    lib = oracle.load()
    assert lib.ref_f16_to_f32(0x3C00) == 1.0
    assert lib.ref_f16_to_f32(0xC000) == -2.0
    assert lib.ref_f16_to_f32(0x7C00) == float("inf")
    assert lib.ref_f16_to_f32(0x0000) == 0.0
    # subnormal 0x0001: the reference counts its 10 normalising shifts up into the
    # exponent: field (10 + 1) + 112 = 123 -> 2^-4 (not 2^-24)
    assert lib.ref_f16_to_f32(0x0001) == 0.0625
    assert lib.ref_f32_to_f16_trunc(np.float32(1.0)) == 0x3C00
    assert lib.ref_f32_to_f16_trunc(np.float32(1e-6)) == 0x0000  # flush to zero
    assert lib.ref_f32_to_f16_trunc(np.float32(70000.0)) == 0x7C00


def test_q4_matvec_interleaved_layout(oracle):
    # one row, 32 columns: nibble byte j holds elements 2j (low) and 2j+1 (high)
    vec = np.arange(32, dtype=np.float32) * 0.25
    q = np.array([(j % 16) for j in range(32)], np.uint8)  # value = q - 8
    block = np.zeros(18, np.uint8)
    block[0], block[1] = 0x00, 0x38  # fp16 0.5
    block[2:] = q[0::2] | (q[1::2] << 4)
    y = oracle.matvec_q4(block, vec, 1, 32)
    acc = np.float32(0)
    for j in range(32):
        acc = np.float32(acc + np.float32(np.float32((int(q[j]) - 8) * np.float32(0.5)) * vec[j]))
    assert y[0] == acc
    y64 = oracle.matvec_q4(block, vec, 1, 32, f64=True)
    assert abs(y64[0] - sum((int(q[j]) - 8) * 0.5 * float(vec[j]) for j in range(32))) < 1e-9


def test_f64_variant_matches_on_small_rows(oracle):
    rng = np.random.default_rng(3)
    for _ in range(50):
        x = rng.standard_normal(64).astype(np.float32) * 3
        for K in (0, 10):
            u = rng.random()
            t32, tr32, _, _ = oracle.sample(x, P(oracle, 0.8, K, 0.9), 30.0, u, F32)
            t64, tr64, _, _ = oracle.sample(x, P(oracle, 0.8, K, 0.9), 30.0, u, F64)
            if min(tr32["boundary"], tr64["boundary"]) > 1e-6:
                assert t32 == t64
