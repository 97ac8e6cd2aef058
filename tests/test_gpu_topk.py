"""GPU parity of the top-K path (configs C1, C2, C5 of BASELINE.json) through
the C ABI, against the oracle's fp32 transcription of DoSample."""
import numpy as np
import pytest

import synth
from gpu_util import BF16, F32, check_topk_rows, run_gpu

pytestmark = pytest.mark.gpu
CAP = 30.0


@pytest.fixture(scope="module")
def c1_rows():
    return np.stack([synth.c1_logits(s) for s in range(1000)]), synth.uniforms(1000, synth.SEEDS["c1"])


def test_c1_batched_1000_steps(sampler, torch_cuda, oracle, g4, c1_rows):
    x, u = c1_rows
    p = g4.make_params(1.0, 64, 0.95)
    res = run_gpu(sampler, torch_cuda, x, F32, p, CAP, u, cand_stride=64)
    st = check_topk_rows(oracle, x, F32, p, CAP, u, res)
    print("C1 batched:", st)
    assert st["rows"] == 1000


def test_c1_single_row_steps(sampler, torch_cuda, oracle, g4, c1_rows):
    # one call per decode step, as TModel.Generate does (B = 1: the cluster kernel)
    x, u = c1_rows
    p = g4.make_params(1.0, 64, 0.95)
    tot = {"boundary": 0}
    for s in range(200):
        res = run_gpu(sampler, torch_cuda, x[s:s + 1], F32, p, CAP, u[s:s + 1], cand_stride=64)
        st = check_topk_rows(oracle, x[s:s + 1], F32, p, CAP, u[s:s + 1], res)
        tot["boundary"] += st["boundary"]
    print("C1 single-row:", tot)


def test_c1_greedy(sampler, torch_cuda, oracle, g4, c1_rows):
    x, u = c1_rows
    p = g4.make_params(0.0, 64, 0.95)
    res = run_gpu(sampler, torch_cuda, x[:300], F32, p, CAP, u[:300], cand_stride=64)
    check_topk_rows(oracle, x[:300], F32, p, CAP, u[:300], res)
    assert (res["flags"] & g4.ROW_GREEDY).all()
    np.testing.assert_array_equal(res["tokens"], np.argmax(x[:300], axis=1))


def test_c2_student_t(sampler, torch_cuda, oracle, g4):
    for step in range(2):
        x = synth.c2_logits(32, step=step)
        u = synth.uniforms(32, synth.SEEDS["c2"], step)
        p = g4.make_params(0.7, 40, 0.9)
        res = run_gpu(sampler, torch_cuda, x, F32, p, CAP, u, cand_stride=40)
        st = check_topk_rows(oracle, x, F32, p, CAP, u, res)
        print("C2:", st)


def test_c5_per_row_params(sampler, torch_cuda, oracle, g4):
    x = synth.c5_logits(192)
    prm = synth.c5_params(192)
    u = synth.uniforms(192, synth.SEEDS["c5"])
    res = run_gpu(sampler, torch_cuda, x, F32, prm, CAP, u, cand_stride=200)
    st = check_topk_rows(oracle, x, F32, prm, CAP, u, res)
    print("C5 rows:", st)


def test_bf16_topk(sampler, torch_cuda, oracle, g4):
    xb = synth.c3_logits(16)
    u = synth.uniforms(16, 77)
    for K in (1, 40, 256):
        p = g4.make_params(0.8, K, 0.9)
        res = run_gpu(sampler, torch_cuda, xb, BF16, p, CAP, u, cand_stride=K)
        check_topk_rows(oracle, xb, BF16, p, CAP, u, res)


def test_large_k_path(sampler, torch_cuda, oracle, g4):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((3, 20000)) * 2).astype(np.float32)
    u = rng.random(3)
    for K in (257, 1000, 19999):
        p = g4.make_params(1.1, K, 0.97)
        res = run_gpu(sampler, torch_cuda, x, F32, p, CAP, u, cand_stride=K)
        check_topk_rows(oracle, x, F32, p, CAP, u, res)


def test_large_k_full_vocab_row(sampler, torch_cuda, oracle, g4):
    x = synth.c1_logits(3)[None, :]
    u = np.array([0.61])
    p = g4.make_params(1.0, 300, 0.95)
    res = run_gpu(sampler, torch_cuda, x, F32, p, CAP, u, cand_stride=300)
    check_topk_rows(oracle, x, F32, p, CAP, u, res)


def test_host_form_matches_device_form(sampler, torch_cuda, oracle, g4, c1_rows):
    x, u = c1_rows
    p = g4.make_params(1.0, 64, 0.95)
    dev = run_gpu(sampler, torch_cuda, x[:64], F32, p, CAP, u[:64])["tokens"]
    s2 = g4.Sampler(0, 64, 262144)
    host = s2.sample_host(np.ascontiguousarray(x[:64]), F32, p, CAP, u[:64])
    s2.close()
    np.testing.assert_array_equal(dev, host)
