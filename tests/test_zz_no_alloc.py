"""g4s_sample_topk_noalloc: top-K sampling that allocates nothing.

Some callers cannot call cudaMalloc when they sample (a host that forbids
allocations after start-up, a decode loop inside a memory pool it does not
own), so they cannot create a g4s_ctx.  This entry point takes its scratch from
a fixed array inside the library instead.  The GPU test checks it against
g4s_sample, the allocating entry point, and against the CPU oracle, call after
call: the calls share the static scratch, so each must leave it ready for the
next.  Tokens on the top-K path are compared exactly, the tolerance every
top-K test here uses, and device free memory must not move across a call.
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
def test_noalloc_matches_sample_call_after_call(g4, torch_cuda, oracle):
    torch = torch_cuda
    lib = g4.load()
    V = synth.V
    s = g4.Sampler(0, 32, V)
    # (rows, dtype, top_k, start offset in elements, row stride padding):
    # small- and big-chunk configurations, both dtypes, and rows that are not
    # 16-byte aligned or not contiguous (the kernels' scalar-load variants)
    calls = [(1, g4.F32, 64, 0, 0), (16, g4.F32, 40, 0, 0), (4, g4.BF16, 64, 0, 0), (1, g4.F32, 64, 0, 0),
             (3, g4.F32, 20, 1, 3), (2, g4.BF16, 64, 3, 5)]
    try:
        for n, (B, dt, K, off, pad) in enumerate(calls):
            if dt == g4.F32:
                x = np.stack([synth.c1_logits(1000 + 37 * n + i) for i in range(B)])
            else:
                x = synth.c3_logits(B, step=n)
            stride = V + pad
            host = np.zeros(B * stride + off, dtype=x.dtype)
            host[off:].reshape(B, stride)[:, :V] = x
            dx = torch.from_numpy(host.view(np.int16) if dt == g4.BF16 else host).cuda()
            ptr = dx.data_ptr() + off * (2 if dt == g4.BF16 else 4)
            u = synth.uniforms(B, 4242, n)
            du = torch.from_numpy(u).cuda()
            want = torch.full((B,), -5, dtype=torch.int32, device="cuda")
            got = torch.full((B,), -6, dtype=torch.int32, device="cuda")
            p = g4.make_params(1.0, K, 0.95)
            torch.cuda.synchronize()
            s.sample(ptr, dt, B, V, stride, p, 30.0, du.data_ptr(), want.data_ptr())
            torch.cuda.synchronize()
            # two calls per configuration: the first may make the driver load
            # device code it had not needed yet (kernels are loaded on first
            # use, the static array with them); the second must leave device
            # memory exactly as it was
            for rep in range(2):
                free_before = torch.cuda.mem_get_info()[0]
                rc = _noalloc(lib, ptr, dt, B, V, stride, p, 30.0, du.data_ptr(), got.data_ptr())
                assert rc == g4.OK, lib.g4s_last_error(None)
                torch.cuda.synchronize()
                free_now = torch.cuda.mem_get_info()[0]
                if rep == 1:
                    assert free_now == free_before, (n, free_before, free_now)
            g = got.cpu().numpy()
            np.testing.assert_array_equal(g, want.cpu().numpy(), err_msg=f"call {n}")
            assert (g >= 0).all()
            # and directly against the oracle's DoSample transcription
            for r in range(B):
                xr = oracle.as_f32(x[r], dt)
                tok, tr, _, _ = oracle.sample(xr, oracle.params(1.0, K, 0.95), 30.0, u[r], oracle.VARIANT_F32,
                                              oracle.TIE_LOWER)
                assert g[r] == tok or tr["boundary"] < 1e-6, (n, r, g[r], tok)
    finally:
        s.close()
