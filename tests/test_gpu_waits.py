"""Bounded waits that run out, made to happen on purpose and safely.

The streaming top-K pass (rows >= 64) waits for each bulk-copied tile on an
mbarrier with a poll limit.  g4s_set_wait_limit(ctx, n) makes every such wait
give up after n non-blocking polls, which the first tile of a CTA cannot meet
(its copy takes about a microsecond).  The kernel must then stop refilling its
ring, wait for the copies it already issued with its normal limit (so nothing
lands in shared memory after it exits), set the device error flag and return.
The host reads the flag once through g4s_device_status (G4S_ERR_TIMEOUT), and
the next call with the normal limits is correct again.  No wait here is left
without an end: the copies it waits for are real and complete.
"""
import numpy as np
import pytest

import synth
from gpu_util import F32, check_topk_rows, run_gpu

pytestmark = pytest.mark.gpu
CAP = 30.0


def test_stream_wait_timeout_reported_once_then_recovers(g4, torch_cuda, oracle):
    torch = torch_cuda
    V, B = synth.V, 64  # 64 aligned fp32 rows: the streaming top-K pass
    x = synth.c5_logits(rows=B, step=11)
    u = synth.uniforms(B, 0x7A17)
    p = g4.make_params(1.0, 64, 0.95)
    with g4.Sampler(0, B, V) as s:
        lib = s.lib
        base = run_gpu(s, torch, x, F32, p, CAP, u, cand_stride=64)
        assert lib.g4s_device_status(s.h) == g4.OK, s.last_error()
        check_topk_rows(oracle, x[:8], F32, p, CAP, u[:8], {k: v[:8] for k, v in base.items()})

        assert lib.g4s_set_wait_limit(s.h, 1) == g4.OK
        run_gpu(s, torch, x, F32, p, CAP, u)  # returns; its tokens are invalid
        assert lib.g4s_device_status(s.h) == g4.ERR_TIMEOUT
        assert "bounded wait" in s.last_error()
        assert lib.g4s_device_status(s.h) == g4.OK  # reported once, then cleared

        assert lib.g4s_set_wait_limit(s.h, 0) == g4.OK
        again = run_gpu(s, torch, x, F32, p, CAP, u, cand_stride=64)
        assert lib.g4s_device_status(s.h) == g4.OK, s.last_error()
        np.testing.assert_array_equal(again["tokens"], base["tokens"])
        np.testing.assert_array_equal(again["cand_ids"], base["cand_ids"])
