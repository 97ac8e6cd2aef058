"""Vocabulary-sharded mode on the GPU through the C ABI.

Ranks are emulated on one GPU: each slice goes through g4s_shard_lists into
its slot of a [W][rows][256] buffer (what the all-gather produces), then
g4s_shard_merge samples.  Tokens must equal g4s_sample on the whole rows (the
top-K path is bit-exact) and the oracle.  With two or more GPUs the NCCL form
(g4s_shard_init / g4s_shard_sample) runs as two processes as well."""
import os

import numpy as np
import pytest

import synth
from gpu_util import BF16, F32, check_topk_rows

pytestmark = pytest.mark.gpu
CAP = 30.0


def _emulated(g4, s, torch, x_dev, dtype, rows, V, prm, u_dev, world):
    esize = 4 if dtype == F32 else 2
    lists = torch.zeros((world, rows, g4.SHARD_LIST), dtype=torch.int64, device="cuda")
    counts = torch.zeros((world, rows), dtype=torch.int32, device="cuda")
    for r, (lo, hi) in enumerate(g4.shard_slices(V, world)):
        s.shard_lists(x_dev.data_ptr() + lo * esize, dtype, rows, hi - lo, V, lo, V, prm,
                      lists[r].data_ptr(), counts[r].data_ptr())
    out = torch.full((rows,), -3, dtype=torch.int32, device="cuda")
    s.shard_merge(lists.data_ptr(), counts.data_ptr(), world, rows, V, prm, CAP, u_dev.data_ptr(), out.data_ptr())
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_emulated_shards_match_unsharded(g4, torch_cuda, oracle, world):
    torch = torch_cuda
    V, rows = 262144, 48
    x = synth.c5_logits(rows, step=world)
    prm = synth.c5_params(rows)
    u = synth.uniforms(rows, 0xC5, world)
    s = g4.Sampler(0, 256, V)
    try:
        xd = torch.from_numpy(x).cuda()
        ud = torch.from_numpy(u).cuda()
        got = _emulated(g4, s, torch, xd, F32, rows, V, prm, ud, world)
        want = torch.full((rows,), -4, dtype=torch.int32, device="cuda")
        s.sample(xd.data_ptr(), F32, rows, V, V, prm, CAP, ud.data_ptr(), want.data_ptr())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got, want.cpu().numpy())
        pick = np.arange(0, rows, 6)
        check_topk_rows(oracle, x[pick], F32, [prm[i] for i in pick], CAP, u[pick], {"tokens": got[pick]})
    finally:
        s.close()


def test_emulated_shards_bf16_and_ties(g4, torch_cuda, oracle):
    torch = torch_cuda
    V, rows, world = 262144, 6, 4
    xb = synth.c3_logits(rows, step=9)
    xb[:, 65530:65545] = xb[0, 7]  # equal values across the first slice boundary
    prm = [(1.0, 64, 0.95), (0.7, 20, 0.9), (0.0, 64, 0.9), (1.3, 200, 0.8), (1.0, 1, 0.5), (0.9, 128, 1.0)]
    u = synth.uniforms(rows, 0xB5)
    s = g4.Sampler(0, 64, V)
    try:
        xd = torch.from_numpy(xb.view(np.int16)).cuda()
        ud = torch.from_numpy(u).cuda()
        got = _emulated(g4, s, torch, xd, BF16, rows, V, prm, ud, world)
        check_topk_rows(oracle, xb, BF16, prm, CAP, u, {"tokens": got})
    finally:
        s.close()


def test_shard_rejects_full_vocab_rows(g4, torch_cuda):
    torch = torch_cuda
    s = g4.Sampler(0, 8, 262144)
    try:
        buf = torch.zeros(8 * 262144, device="cuda")
        lists = torch.zeros((8, g4.SHARD_LIST), dtype=torch.int64, device="cuda")
        counts = torch.zeros(8, dtype=torch.int32, device="cuda")
        rc = s.shard_lists(buf.data_ptr(), F32, 8, 131072, 262144, 0, 262144, g4.make_params(1.0, 0, 0.9),
                           lists.data_ptr(), counts.data_ptr(), check=False)
        assert rc == g4.ERR_ARG and "row split" in s.last_error()
    finally:
        s.close()


def _nccl_rank(rank, world, uid_path, x, prm, u, out_path):
    import torch

    import g4sampler as g4

    torch.cuda.set_device(rank)
    V, rows = x.shape[1], x.shape[0]
    lo, hi = g4.shard_slices(V, world)[rank]
    s = g4.Sampler(rank, rows, V)
    for _ in range(600):
        if os.path.exists(uid_path):
            break
        import time

        time.sleep(0.05)
    uid = open(uid_path, "rb").read()
    s.shard_init(world, rank, V, uid)
    xs = torch.from_numpy(np.ascontiguousarray(x[:, lo:hi])).cuda()
    ud = torch.from_numpy(u).cuda()
    out = torch.full((rows,), -2, dtype=torch.int32, device="cuda")
    s.shard_sample(xs.data_ptr(), F32, rows, hi - lo, prm, CAP, ud.data_ptr(), out.data_ptr())
    torch.cuda.synchronize()
    np.save(out_path % rank, out.cpu().numpy())
    s.close()


def test_nccl_two_ranks(g4, torch_cuda, oracle, tmp_path):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    V, rows, world = 262144, 16, 2
    x = synth.c5_logits(rows, step=77)
    prm = synth.c5_params(rows)
    u = synth.uniforms(rows, 0x77)
    uid_path = str(tmp_path / "uid.bin")
    open(uid_path + ".tmp", "wb").write(g4.shard_unique_id())
    os.rename(uid_path + ".tmp", uid_path)
    out_path = str(tmp_path / "tok%d.npy")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_nccl_rank, args=(world, uid_path, x, prm, u, out_path), nprocs=world, join=True)
    t0, t1 = np.load(out_path % 0), np.load(out_path % 1)
    np.testing.assert_array_equal(t0, t1)
    check_topk_rows(oracle, x, F32, prm, CAP, u, {"tokens": t0})
