"""GPU parity of the full-vocabulary path (the
headline bandwidth-bound pass) through the C ABI, against the oracle's fp64
restatement of DoSampleTopP + CpuSoftmaxF32 + CpuLogitSoftcap."""
import numpy as np
import pytest

import synth
from gpu_util import BF16, F32, check_full_rows, run_gpu

pytestmark = pytest.mark.gpu
CAP = 30.0


@pytest.fixture(scope="module")
def c3_rows():
    return synth.c3_logits(32), synth.uniforms(32, synth.SEEDS["c3"])


def test_c3_tokens_and_probabilities(sampler, torch_cuda, oracle, g4, c3_rows):
    xb, u = c3_rows
    p = g4.make_params(1.0, 0, 0.95)
    res = run_gpu(sampler, torch_cuda, xb, BF16, p, CAP, u, full_probs=True)
    assert (res["flags"] & g4.ROW_FULL_PATH).all()
    st = check_full_rows(oracle, xb, BF16, p, CAP, u, res)
    print("C3:", st)
    assert st["rows"] == 32


def test_c3_greedy(sampler, torch_cuda, oracle, g4, c3_rows):
    xb, u = c3_rows
    p = g4.make_params(0.0, 0, 0.95)
    res = run_gpu(sampler, torch_cuda, xb, BF16, p, CAP, u)
    check_full_rows(oracle, xb, BF16, p, CAP, u, res, check_probs=False)


def test_full_path_fp32_with_temperature(sampler, torch_cuda, oracle, g4):
    x = np.stack([synth.c1_logits(s) for s in range(8)])
    u = synth.uniforms(8, 99)
    for T, K in ((0.7, 0), (1.3, 262144), (1.0, -3)):
        p = g4.make_params(T, K, 0.9)
        res = run_gpu(sampler, torch_cuda, x, F32, p, CAP, u, full_probs=True)
        check_full_rows(oracle, x, F32, p, CAP, u, res)


def test_full_path_small_batch_kernel(sampler, torch_cuda, oracle, g4, c3_rows):
    # B = 1..4 selects the small-chunk configuration
    xb, u = c3_rows
    p = g4.make_params(1.0, 0, 0.95)
    for B in (1, 4):
        res = run_gpu(sampler, torch_cuda, xb[:B], BF16, p, CAP, u[:B], full_probs=True)
        check_full_rows(oracle, xb[:B], BF16, p, CAP, u[:B], res)


def test_full_path_threshold_sweep(sampler, torch_cuda, oracle, g4, c3_rows):
    # many draws on the same row: exercises chunk / sub-range / element location
    xb, _ = c3_rows
    rows = np.repeat(xb[:1], 64, axis=0)
    u = np.linspace(0.0, 0.999999, 64)
    p = g4.make_params(1.0, 0, 1.0)
    res = run_gpu(sampler, torch_cuda, rows, BF16, p, CAP, u)
    st = check_full_rows(oracle, rows, BF16, p, CAP, u, res, check_probs=False)
    print("sweep:", st)
    assert np.all(np.diff(res["tokens"]) >= 0)  # index-order CDF: monotone in u


def test_c3_full_size_batch(sampler, torch_cuda, oracle, g4):
    # the benchmark configuration (256 x 262144 bf16); oracle on a sample of rows
    xb = synth.c3_logits(256, step=1)
    u = synth.uniforms(256, synth.SEEDS["c3"], 1)
    p = g4.make_params(1.0, 0, 0.95)
    res = run_gpu(sampler, torch_cuda, xb, BF16, p, CAP, u)
    pick = np.arange(0, 256, 16)
    sub = {k: v[pick] for k, v in res.items()}
    st = check_full_rows(oracle, xb[pick], BF16, p, CAP, u[pick], sub, check_probs=False)
    print("C3 full batch sample:", st)
    assert ((res["tokens"] >= 0) & (res["tokens"] < 262144)).all()


def test_full_path_general_items_bf16(sampler, torch_cuda, oracle, g4):
    # bf16 rows on the aligned (shared-memory ring) path with items the fast
    # polynomial cannot take: a NaN, a logit beyond +cap, many below -cap.
    # The streaming pass flags them and redoes them on the general path.
    V = 262144
    xb = synth.c3_logits(5, step=11)
    rng = np.random.default_rng(12)
    xb[0, rng.choice(V, 7, replace=False)] = 0x7FC0                       # NaN
    xb[1, rng.choice(V, 3, replace=False)] = synth.f32_to_bf16_rne(np.float32([45.0]))[0]
    xb[2, ::97] = synth.f32_to_bf16_rne(np.float32([-60.0]))[0]           # every item
    xb[3, :5] = synth.f32_to_bf16_rne(np.float32([-31.0]))[0]
    u = synth.uniforms(5, 1234)
    for T in (1.0, 0.8):
        p = g4.make_params(T, 0, 0.95)
        res = run_gpu(sampler, torch_cuda, xb, BF16, p, CAP, u, full_probs=True)
        st = check_full_rows(oracle, xb, BF16, p, CAP, u, res)
        assert st["rows"] == 5
    # greedy rows take the same items
    p = g4.make_params(0.0, 0, 0.95)
    res = run_gpu(sampler, torch_cuda, xb, BF16, p, CAP, u)
    check_full_rows(oracle, xb, BF16, p, CAP, u, res, check_probs=False)
