"""Edge cases through the C ABI: tiny and ragged vocabularies, unaligned and
strided rows, ties, masked (-inf / <= -1e30) logits, empty rows, NaN policy,
degenerate draws, softcap disabled, and argument errors."""
import numpy as np
import pytest

import synth
from gpu_util import BF16, F32, check_full_rows, check_topk_rows, run_gpu

pytestmark = pytest.mark.gpu
CAP = 30.0


def _both(sampler, torch, oracle, x, dtype, params, cap, u, **kw):
    """Route rows to the right checker by their path."""
    import g4sampler as g4

    V = x.shape[1]
    K = params.top_k if isinstance(params, g4.Params) else None
    full = K is not None and (K <= 0 or K >= V)
    res = run_gpu(sampler, torch, x, dtype, params, cap, u,
                  cand_stride=0 if full else max(1, min(K, 4096)), full_probs=full, **kw)
    if full:
        return check_full_rows(oracle, x, dtype, params, cap, u, res)
    return check_topk_rows(oracle, x, dtype, params, cap, u, res)


@pytest.mark.parametrize("V", [1, 2, 3, 5, 7, 8, 13, 100, 1000, 2047, 2048, 2049, 8191, 8193, 20011])
def test_ragged_vocab_sizes(sampler, torch_cuda, oracle, g4, V):
    rng = np.random.default_rng(V)
    x = (rng.standard_normal((3, V)) * 3).astype(np.float32)
    u = rng.random(3)
    for K in sorted({0, 1, 2, min(40, V - 1), V - 1, V}):
        if K < 0:
            continue
        _both(sampler, torch_cuda, oracle, x, F32, g4.make_params(0.9, K, 0.9), CAP, u)


@pytest.mark.parametrize("offset,stride_pad", [(1, 0), (0, 3), (3, 5)])
def test_unaligned_and_strided_rows(sampler, torch_cuda, oracle, g4, offset, stride_pad):
    rng = np.random.default_rng(offset * 10 + stride_pad)
    V = 5000
    x = (rng.standard_normal((4, V)) * 3).astype(np.float32)
    u = rng.random(4)
    for K in (0, 50):
        p = g4.make_params(1.0, K, 0.95)
        _both(sampler, torch_cuda, oracle, x, F32, p, CAP, u, row_stride=V + stride_pad, offset_elems=offset)
    xb = (rng.standard_normal((4, V)) * 3).astype(np.float32).view(np.uint32)
    xb = (xb >> 16).astype(np.uint16)
    for K in (0, 50):
        p = g4.make_params(1.0, K, 0.95)
        _both(sampler, torch_cuda, oracle, xb, BF16, p, CAP, u, row_stride=V + stride_pad, offset_elems=offset)


def test_heavy_ties(sampler, torch_cuda, oracle, g4):
    # constant rows, few distinct values: the K-th place is tied across chunks
    V = 262144
    rng = np.random.default_rng(1)
    x = np.stack([np.zeros(V, np.float32), rng.integers(0, 3, V).astype(np.float32),
                  np.repeat(np.arange(64, dtype=np.float32), V // 64)])
    u = np.array([0.3, 0.6, 0.9])
    for K in (1, 7, 64, 200, 256):
        st = _both(sampler, torch_cuda, oracle, x, F32, g4.make_params(1.0, K, 0.95), CAP, u)
        print(K, st)
    _both(sampler, torch_cuda, oracle, x, F32, g4.make_params(1.0, 0, 0.95), CAP, u)


def test_masked_logits_and_short_rows(sampler, torch_cuda, oracle, g4):
    V = 30000
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((4, V)) * 3).astype(np.float32)
    x[0, :] = -np.inf
    x[0, [5, 777, 29999]] = [1.0, 2.0, 3.0]     # only 3 candidates for K = 64
    x[1, :] = -1e30                               # exactly -1e30 is not a candidate
    x[1, 12345] = -1e29
    x[2, ::2] = -2e30
    x[3, :] = -np.inf                             # no candidate at all: token -1
    u = rng.random(4)
    p = g4.make_params(1.0, 64, 0.95)
    res = run_gpu(sampler, torch_cuda, x, F32, p, CAP, u, cand_stride=64)
    check_topk_rows(oracle, x, F32, p, CAP, u, res)
    assert res["tokens"][3] == -1 and res["flags"][3] & g4.ROW_EMPTY
    # the full path keeps masked logits (softcap maps -inf to -cap)
    _both(sampler, torch_cuda, oracle, x, F32, g4.make_params(1.0, 0, 0.95), CAP, u)


def test_nan_policy(sampler, torch_cuda, oracle, g4):
    V = 4096
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((2, V)) * 3).astype(np.float32)
    x[:, rng.choice(V, 100, replace=False)] = np.nan
    u = rng.random(2)
    for K in (0, 20):
        _both(sampler, torch_cuda, oracle, x, F32, g4.make_params(1.0, K, 0.95), CAP, u)


def test_degenerate_draws(sampler, torch_cuda, oracle, g4):
    V = 50000
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((4, V)) * 3).astype(np.float32)
    for K in (0, 64):
        # u = 0 picks the first candidate in id order; top_p > 1 falls back to argmax
        _both(sampler, torch_cuda, oracle, x, F32, g4.make_params(1.0, K, 0.95), CAP, np.zeros(4))
        st = _both(sampler, torch_cuda, oracle, x, F32, g4.make_params(1.0, K, 1.5), CAP,
                   np.array([0.99, 0.999, 0.7, 0.9999]))
        print("fallback", K, st)
        _both(sampler, torch_cuda, oracle, x, F32, g4.make_params(1.0, K, 0.0), CAP, rng.random(4))


def test_softcap_disabled_and_extremes(sampler, torch_cuda, oracle, g4):
    V = 9000
    rng = np.random.default_rng(6)
    x = (rng.standard_normal((3, V)) * 40).astype(np.float32)   # |q| > 1 hits the wide tanh branch
    x[0, 7] = np.inf
    x[2, :10] = 1e-30                                            # tiny values
    u = rng.random(3)
    for cap in (CAP, 0.0):
        for K in (0, 30):
            rows = x if cap > 0 or K > 0 else x[1:]             # +inf without softcap: outside the contract
            _both(sampler, torch_cuda, oracle, rows, F32, g4.make_params(1.0, K, 0.9), cap, u[:rows.shape[0]])


def test_per_row_mixed_paths(sampler, torch_cuda, oracle, g4):
    V = 40000
    rng = np.random.default_rng(8)
    x = (rng.standard_normal((6, V)) * 3).astype(np.float32)
    prm = [(1.0, 0, 0.9), (0.5, 64, 0.8), (0.0, 10, 0.9), (1.2, 300, 0.95), (1.0, V, 0.7), (0.0, 0, 0.5)]
    u = rng.random(6)
    res = run_gpu(sampler, torch_cuda, x, F32, prm, CAP, u, cand_stride=300)
    for r, (T, K, P) in enumerate(prm):
        one = {k: v[r:r + 1] for k, v in res.items()}
        if K <= 0 or K >= V:
            one.pop("cand_ids"), one.pop("cand_probs")
            check_full_rows(oracle, x[r:r + 1], F32, [prm[r]], CAP, u[r:r + 1], one, check_probs=False)
        else:
            check_topk_rows(oracle, x[r:r + 1], F32, [prm[r]], CAP, u[r:r + 1], one)


def test_repeated_calls_reuse_workspace(sampler, torch_cuda, oracle, g4):
    # counters left by one call must not disturb the next (different shapes too)
    rng = np.random.default_rng(9)
    for i in range(6):
        V = [262144, 7000, 262144, 100, 50000, 262144][i]
        B = [2, 5, 64, 1, 9, 1][i]
        x = (rng.standard_normal((B, V)) * 3).astype(np.float32)
        u = rng.random(B)
        _both(sampler, torch_cuda, oracle, x, F32, g4.make_params(1.0, [64, 0][i % 2], 0.95), CAP, u)


def test_argument_errors(sampler, torch_cuda, g4):
    import torch

    x = torch.zeros((2, 100), device="cuda")
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    u = torch.zeros(2, dtype=torch.float64, device="cuda")
    p = g4.make_params()
    assert sampler.sample(x.data_ptr(), 7, 2, 100, 100, p, CAP, u.data_ptr(), out.data_ptr(), check=False) == g4.ERR_ARG
    assert sampler.sample(x.data_ptr(), F32, 2, 100, 99, p, CAP, u.data_ptr(), out.data_ptr(), check=False) == g4.ERR_ARG
    assert sampler.sample(x.data_ptr(), F32, 2000, 100, 100, p, CAP, u.data_ptr(), out.data_ptr(), check=False) == g4.ERR_CAPACITY
    assert sampler.sample(x.data_ptr(), F32, 2, 100, 100, p, CAP, 0, out.data_ptr(), check=False) == g4.ERR_ARG
    assert "u is NULL" in sampler.last_error()
    # greedy rows need no draws
    pg = g4.make_params(0.0, 5, 0.9)
    assert sampler.sample(x.data_ptr(), F32, 2, 100, 100, pg, CAP, 0, out.data_ptr(), check=False) == g4.OK
    torch.cuda.synchronize()


@pytest.mark.parametrize("K", [128, 200])
def test_single_row_cluster_merge_paths(sampler, torch_cuda, oracle, g4, K):
    # Rows of a small batch with top_k <= 128 take the one-cluster-per-row
    # kernel (16 slices of 16384 ids); K = 200 takes the chunked grid.  Row 0
    # interleaves the slices' top entries, so every slice holds many entries at
    # or above the row's bound (the largest pushes, or the exact per-slice
    # fallback); row 1 keeps them apart (few pushes from most slices).
    V = 262144
    x = np.full((2, V), -1e30, dtype=np.float32)
    for c in range(16):
        i = np.arange(K)
        pos = c * 16384 + (i * 37) % 16384
        x[0, pos] = 1.0 + (i * 16 + c) * 1e-3
        x[1, pos] = 1.0 + c + i * 1e-3
    u = np.array([0.37, 0.81])
    for T in (1.0, 0.0):
        _both(sampler, torch_cuda, oracle, x, F32, g4.make_params(T, K, 0.9), CAP, u)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_streaming_topk_batches(sampler, torch_cuda, oracle, g4, dtype):
    # batches of 64 rows or more with aligned rows take the streaming top-K pass
    # (long chunks through a bulk-copy tile ring, a running bound, buffer cuts).
    # Constant rows force the exact radix cut; NaNs, masked and almost empty
    # rows, per-row K from 1 to 256, and a padded row stride with a vocabulary
    # that is not a whole number of vectors (the ragged end of each row's last
    # chunk comes through plain loads).
    rows, V, stride = 80, 262141, 262144
    rng = np.random.default_rng(21)
    x = (rng.standard_normal((rows, V)) * 3).astype(np.float32)
    x[0, :] = 1.5                                             # one value: ties everywhere
    x[1, :] = rng.integers(0, 4, V).astype(np.float32)        # four values
    x[2, rng.choice(V, 500, replace=False)] = np.nan
    x[3, :] = -np.inf
    x[3, [7, 131071, V - 1]] = [2.0, 1.0, 3.0]                # three candidates
    x[4, -5:] = 40.0                                          # the top K in the ragged end
    if dtype == "bf16":
        xd, dt = synth.f32_to_bf16_rne(x), BF16
    else:
        xd, dt = x, F32
    ks = [1, 40, 64, 256, 7]
    prm = [(0.8 if r % 3 else 1.0, ks[r % len(ks)], 0.9) for r in range(rows)]
    u = rng.random(rows)
    res = run_gpu(sampler, torch_cuda, xd, dt, prm, CAP, u, cand_stride=256, row_stride=stride)
    check_topk_rows(oracle, xd, dt, prm, CAP, u, res)
