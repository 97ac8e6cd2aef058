"""Failure handling of the NCCL form of the vocabulary-sharded mode, with the
failure made on the host: a rank that never joins the rendezvous, and a rank
that stops taking part between steps (alive, none of its work in flight) while
its peer runs the next step.  The waiting side must come back with
G4S_ERR_TIMEOUT within its deadline, with the communicator aborted (which ends
its collective kernels waiting on the peer) and the context still usable.
Ranks run as child processes with NVLS off."""
import os
import time

import numpy as np
import pytest

import synth
from gpu_util import F32

pytestmark = pytest.mark.gpu
CAP = 30.0


def _lonely_rank(_, uid_path, out_path):
    import torch

    import g4sampler as g4

    torch.cuda.set_device(0)
    s = g4.Sampler(0, 8, 131072)
    s.shard_set_timeout(2000)
    uid = open(uid_path, "rb").read()
    t0 = time.monotonic()
    rc = s.shard_init(2, 0, 262144, uid, check=False)  # rank 1 never comes
    took = time.monotonic() - t0
    err = s.last_error()
    # the context keeps working unsharded
    x = torch.from_numpy(synth.c5_logits(8, vocab=131072, step=1)).cuda()
    u = torch.from_numpy(synth.uniforms(8, 3)).cuda()
    out = torch.full((8,), -1, dtype=torch.int32, device="cuda")
    s.sample(x.data_ptr(), F32, 8, 131072, 131072, g4.make_params(1.0, 64, 0.95), CAP, u.data_ptr(), out.data_ptr())
    torch.cuda.synchronize()
    ok = bool((out.cpu().numpy() >= 0).all())
    s.close()
    np.save(out_path, np.array([rc, took, ok], dtype=np.float64))
    open(out_path + ".txt", "w").write(err)


def test_init_times_out_when_a_rank_never_joins(g4, torch_cuda, tmp_path):
    import torch.multiprocessing as mp

    uid_path = str(tmp_path / "uid.bin")
    open(uid_path, "wb").write(g4.shard_unique_id())
    out_path = str(tmp_path / "lonely.npy")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_lonely_rank, args=(uid_path, out_path), nprocs=1, join=True)
    rc, took, ok = np.load(out_path)
    assert int(rc) == g4.ERR_TIMEOUT, open(out_path + ".txt").read()
    assert took < 30.0
    assert "did not join" in open(out_path + ".txt").read()
    assert ok


def _stall_rank(rank, world, uid_path, flag_path, out_path, x, prm, u):
    import torch

    import g4sampler as g4

    torch.cuda.set_device(rank)
    V, rows = x.shape[1], x.shape[0]
    lo, hi = g4.shard_slices(V, world)[rank]
    s = g4.Sampler(rank, rows, V)
    s.shard_set_timeout(20000)
    for _ in range(600):
        if os.path.exists(uid_path):
            break
        time.sleep(0.05)
    s.shard_init(world, rank, V, open(uid_path, "rb").read())
    xs = torch.from_numpy(np.ascontiguousarray(x[:, lo:hi])).cuda()
    ud = torch.from_numpy(u).cuda()
    out = torch.full((rows,), -2, dtype=torch.int32, device="cuda")
    res = {}
    # step 1: every rank takes part
    s.shard_sample(xs.data_ptr(), F32, rows, hi - lo, prm, CAP, ud.data_ptr(), out.data_ptr())
    res["wait1"] = s.shard_wait(timeout_ms=20000, check=False)
    res["tok1"] = out.cpu().numpy().copy()
    if rank == 0:
        # step 2 without the peer: the all-gather waits on it until the deadline
        t0 = time.monotonic()
        rc = s.shard_sample(xs.data_ptr(), F32, rows, hi - lo, prm, CAP, ud.data_ptr(), out.data_ptr(), check=False)
        res["sample2"] = rc
        res["wait2"] = s.shard_wait(timeout_ms=3000, check=False) if rc == g4.OK else rc
        res["took2"] = time.monotonic() - t0
        res["err2"] = s.last_error()
        res["wait3"] = s.shard_wait(check=False)  # unsharded now
        open(flag_path, "w").write("aborted")
    else:
        # alive, between steps, nothing in flight; told of the failure on the host
        for _ in range(1200):
            if os.path.exists(flag_path):
                break
            time.sleep(0.05)
        s.shard_abort()
    # the context keeps working unsharded
    xf = torch.from_numpy(x).cuda()
    full = torch.full((rows,), -3, dtype=torch.int32, device="cuda")
    s2 = g4.Sampler(rank, rows, V)
    s2.sample(xf.data_ptr(), F32, rows, V, V, prm, CAP, ud.data_ptr(), full.data_ptr())
    s.sample(xf.data_ptr(), F32, rows, hi - lo, V, prm, CAP, ud.data_ptr(), out.data_ptr())
    torch.cuda.synchronize()
    res["after_ok"] = bool((out.cpu().numpy() >= 0).all())
    res["full"] = full.cpu().numpy()
    s2.close()
    s.close()
    np.save(out_path % rank, np.array([res], dtype=object), allow_pickle=True)


def test_step_times_out_when_a_peer_stalls(g4, torch_cuda, tmp_path):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    V, rows, world = 262144, 16, 2
    x = synth.c5_logits(rows, step=91)
    prm = synth.c5_params(rows)
    u = synth.uniforms(rows, 0x91)
    uid_path = str(tmp_path / "uid.bin")
    open(uid_path + ".tmp", "wb").write(g4.shard_unique_id())
    os.rename(uid_path + ".tmp", uid_path)
    flag_path = str(tmp_path / "aborted.flag")
    out_path = str(tmp_path / "r%d.npy")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_stall_rank, args=(world, uid_path, flag_path, out_path, x, prm, u), nprocs=world, join=True)
    r0 = np.load(out_path % 0, allow_pickle=True)[0]
    r1 = np.load(out_path % 1, allow_pickle=True)[0]
    assert r0["wait1"] == g4.OK and r1["wait1"] == g4.OK
    np.testing.assert_array_equal(r0["tok1"], r1["tok1"])
    np.testing.assert_array_equal(r0["tok1"], r0["full"])  # step 1 equals the unsharded tokens
    assert r0["wait2"] == g4.ERR_TIMEOUT, r0["err2"]
    assert "aborted" in r0["err2"]
    assert r0["took2"] < 20.0
    assert r0["wait3"] == g4.ERR_STATE  # the context left the sharded state
    assert r0["after_ok"] and r1["after_ok"]
