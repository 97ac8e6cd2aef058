"""g4s_sample_topk_noalloc: top-K sampling that allocates nothing.

Some callers cannot call cudaMalloc when they sample (a host that forbids
allocations after start-up, a decode loop inside a memory pool it does not
own), so they cannot create a g4s_ctx.  This entry point takes its scratch from
a fixed array inside the library instead.  The GPU test checks it against
g4s_sample, the allocating entry point, call after call: the calls share the
static scratch, so each must leave it ready for the next.  Tokens on the top-K
path are compared exactly, the tolerance every top-K test here uses.
"""
import ctypes

import numpy as np
import pytest

import synth


def _noalloc(lib, ptr, dtype, rows, vocab, stride, p, cap, u_ptr, out_ptr):
    return lib.g4s_sample_topk_noalloc(ctypes.c_void_p(ptr), dtype, rows, vocab, stride, ctypes.byref(p),
                                       cap, ctypes.c_void_p(u_ptr), ctypes.c_void_p(out_ptr), None)


def test_noalloc_rejects_out_of_contract_calls(g4):
    # argument checks run before any CUDA call
    lib = g4.load()
    p = g4.make_params(1.0, 64, 0.95)
    assert _noalloc(lib, 16, g4.F32, 65, 262144, 262144, p, 30.0, 16, 16) == g4.ERR_CAPACITY
    assert b"static maximum" in lib.g4s_last_error(None)
    assert _noalloc(lib, 16, g4.F32, 1, 262144, 262144, g4.make_params(1.0, 0, 0.95), 30.0, 16, 16) == g4.ERR_ARG
    assert _noalloc(lib, 16, g4.F32, 1, 262144, 262144, g4.make_params(1.0, 300, 0.95), 30.0, 16, 16) == g4.ERR_ARG
    assert _noalloc(lib, 0, g4.F32, 1, 262144, 262144, p, 30.0, 16, 16) == g4.ERR_ARG
    assert _noalloc(lib, 16, g4.F32, 1, 262144, 262144, p, 30.0, 0, 16) == g4.ERR_ARG


@pytest.mark.gpu
def test_noalloc_matches_sample_call_after_call(g4, torch_cuda):
    torch = torch_cuda
    lib = g4.load()
    V = synth.V
    s = g4.Sampler(0, 32, V)
    # (rows, dtype, top_k): small-chunk and big-chunk configurations, both dtypes
    calls = [(1, g4.F32, 64), (16, g4.F32, 40), (4, g4.BF16, 64), (1, g4.F32, 64)]
    try:
        for n, (B, dt, K) in enumerate(calls):
            if dt == g4.F32:
                x = np.stack([synth.c1_logits(1000 + 37 * n + i) for i in range(B)])
                dx = torch.from_numpy(x).cuda()
            else:
                x = synth.c3_logits(B, step=n)
                dx = torch.from_numpy(x.view(np.int16)).cuda()
            u = synth.uniforms(B, 4242, n)
            du = torch.from_numpy(u).cuda()
            want = torch.full((B,), -5, dtype=torch.int32, device="cuda")
            got = torch.full((B,), -6, dtype=torch.int32, device="cuda")
            p = g4.make_params(1.0, K, 0.95)
            torch.cuda.synchronize()
            s.sample(dx.data_ptr(), dt, B, V, V, p, 30.0, du.data_ptr(), want.data_ptr())
            torch.cuda.synchronize()
            rc = _noalloc(lib, dx.data_ptr(), dt, B, V, V, p, 30.0, du.data_ptr(), got.data_ptr())
            assert rc == g4.OK, lib.g4s_last_error(None)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(got.cpu().numpy(), want.cpu().numpy(), err_msg=f"call {n}")
            assert (got >= 0).all()
    finally:
        s.close()
