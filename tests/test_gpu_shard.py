"""Vocabulary-sharded mode on the GPU through the C ABI.

Ranks are emulated on one GPU: each slice goes through g4s_shard_lists into
its slot of a [W][rows][256] buffer (what the all-gather produces), then
g4s_shard_merge samples.  Tokens must equal g4s_sample on the whole rows (the
top-K path is bit-exact) and the oracle.  Full-vocabulary rows add the
resolve phase: each emulated rank has its own context (its slice's item
statistics and its merge's targets), runs lists, merge and
g4s_shard_resolve, and the ranks' outputs are combined by an element-wise max
(the all-reduce).  With two or more GPUs the NCCL form (g4s_shard_init /
g4s_shard_sample) runs as processes as well."""
import os

import numpy as np
import pytest

import synth
from gpu_util import BF16, F32, check_full_rows, check_topk_rows

pytestmark = pytest.mark.gpu
CAP = 30.0


def _emulated(g4, s, torch, x_dev, dtype, rows, V, prm, u_dev, world):
    esize = 4 if dtype == F32 else 2
    lists = torch.zeros((world, rows, g4.SHARD_LIST), dtype=torch.int64, device="cuda")
    counts = torch.zeros((world, rows), dtype=torch.int32, device="cuda")
    for r, (lo, hi) in enumerate(g4.shard_slices(V, world)):
        s.shard_lists(x_dev.data_ptr() + lo * esize, dtype, rows, hi - lo, V, lo, V, prm, CAP,
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


def _emulated_full(g4, torch, x_dev, dtype, rows, V, prm, u_dev, world, cap=CAP):
    """Every emulated rank on its own context: lists, all-gather (a copy into
    the shared buffer), merge, resolve; then the max over the ranks."""
    esize = 4 if dtype == F32 else 2
    sl = g4.shard_slices(V, world)
    ctxs = [g4.Sampler(0, rows, max(hi - lo for lo, hi in sl)) for _ in range(world)]
    try:
        lists = torch.zeros((world, rows, g4.SHARD_LIST), dtype=torch.int64, device="cuda")
        counts = torch.zeros((world, rows), dtype=torch.int32, device="cuda")
        for r, (lo, hi) in enumerate(sl):
            ctxs[r].shard_lists(x_dev.data_ptr() + lo * esize, dtype, rows, hi - lo, V, lo, V, prm, cap,
                                lists[r].data_ptr(), counts[r].data_ptr())
        toks = torch.full((world, rows), -3, dtype=torch.int32, device="cuda")
        tprob = torch.full((world, rows), -1.0, dtype=torch.float32, device="cuda")
        flags = torch.zeros((world, rows), dtype=torch.int32, device="cuda")
        for r, (lo, hi) in enumerate(sl):
            o = g4.Outputs()
            o.token_prob = tprob[r].data_ptr()
            o.row_flags = flags[r].data_ptr()
            ctxs[r].shard_merge(lists.data_ptr(), counts.data_ptr(), world, rows, V, prm, cap, u_dev.data_ptr(),
                                toks[r].data_ptr(), outputs=o)
            ctxs[r].shard_resolve(x_dev.data_ptr() + lo * esize, dtype, rows, hi - lo, V, lo, r, prm, cap,
                                  u_dev.data_ptr(), toks[r].data_ptr(), outputs=o)
        torch.cuda.synchronize()
        return (toks.max(0).values.cpu().numpy(), tprob.max(0).values.cpu().numpy(), flags.cpu().numpy(),
                toks.cpu().numpy(), counts.cpu().numpy())
    finally:
        for c in ctxs:
            c.close()


def _unsharded(g4, torch, x_dev, dtype, rows, V, prm, u_dev):
    s = g4.Sampler(0, rows, V)
    try:
        out = torch.full((rows,), -4, dtype=torch.int32, device="cuda")
        tp = torch.zeros(rows, dtype=torch.float32, device="cuda")
        o = g4.Outputs()
        o.token_prob = tp.data_ptr()
        s.sample(x_dev.data_ptr(), dtype, rows, V, V, prm, CAP, u_dev.data_ptr(), out.data_ptr(), outputs=o)
        torch.cuda.synchronize()
        return out.cpu().numpy(), tp.cpu().numpy()
    finally:
        s.close()


def _full_params(rows):
    # full-vocabulary draws (top_k 0 and top_k >= vocab), greedy full rows and
    # top-K rows in one batch
    base = [(1.0, 0, 0.95), (0.8, 0, 1.0), (0.0, 0, 0.9), (1.2, 262144, 0.9), (1.0, 64, 0.95), (0.6, 0, 0.5),
            (1.5, 0, 0.99), (0.9, 20, 0.9)]
    return [base[r % len(base)] for r in range(rows)]


@pytest.mark.parametrize("world,dtype", [(2, BF16), (4, BF16), (8, BF16), (2, F32), (8, F32)])
def test_emulated_full_rows_match_unsharded(g4, torch_cuda, oracle, world, dtype):
    torch = torch_cuda
    V, rows = 262144, 24
    if dtype == BF16:
        x = synth.c3_logits(rows, step=world)
        xd = torch.from_numpy(x.view(np.int16)).cuda()
    else:
        x = synth.c5_logits(rows, step=world)
        xd = torch.from_numpy(x).cuda()
    prm = _full_params(rows)
    u = synth.uniforms(rows, 0xF5, world)
    ud = torch.from_numpy(u).cuda()
    got, gprob, flags, per_rank, counts = _emulated_full(g4, torch, xd, dtype, rows, V, prm, ud, world)
    want, wprob = _unsharded(g4, torch, xd, dtype, rows, V, prm, ud)
    full = np.array([K <= 0 or K >= V for _, K, _ in prm])
    draw = np.array([T > 0 for T, _, _ in prm])
    assert (counts[:, full] == -1).all() and (counts[:, ~full] > 0).all()
    # a full draw is written by exactly one rank; the others keep -1
    fd = full & draw
    assert ((per_rank[:, fd] >= 0).sum(0) == 1).all()
    assert (per_rank[:, ~fd] == per_rank[0, ~fd]).all()
    # fp64 summation in another order: a token may differ only at a boundary,
    # which these seeds do not reach
    np.testing.assert_array_equal(got, want)
    np.testing.assert_allclose(gprob[full], wprob[full], rtol=1e-6, atol=0)
    assert (flags[:, full] & g4.ROW_FULL_PATH).all()
    pick = np.flatnonzero(full)[:6]
    st = check_full_rows(oracle, x[pick], dtype, [prm[i] for i in pick], CAP, u[pick], {"tokens": got[pick]},
                         check_probs=False)
    assert st["rows"] == len(pick)


def test_emulated_full_rows_without_softcap_and_peaked(g4, torch_cuda, oracle):
    # softcap 0 (plain logits) on f32 rows with one dominant token per row and
    # rows whose mass sits in the last slice: the crossing shard is the last one
    torch = torch_cuda
    V, rows, world = 262144, 8, 4
    rng = np.random.default_rng(71)
    x = (rng.standard_normal((rows, V)) * 2).astype(np.float32)
    x[0, 5] = 40.0
    x[1, V - 3] = 40.0
    x[2, 200000:] += 6.0
    x[3, :] = 1.0  # uniform row: the draw lands by u alone
    prm = [(1.0, 0, 1.0)] * rows
    u = synth.uniforms(rows, 0x71)
    u[3] = 0.999999
    xd = torch.from_numpy(x).cuda()
    ud = torch.from_numpy(u).cuda()
    got, _, _, _, _ = _emulated_full(g4, torch, xd, F32, rows, V, prm, ud, world, cap=0.0)
    s = g4.Sampler(0, rows, V)
    try:
        out = torch.full((rows,), -4, dtype=torch.int32, device="cuda")
        s.sample(xd.data_ptr(), F32, rows, V, V, prm, 0.0, ud.data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got, out.cpu().numpy())
    finally:
        s.close()
    assert got[0] == 5 and got[1] == V - 3
    check_full_rows(oracle, x, F32, prm, 0.0, u, {"tokens": got}, check_probs=False)


def test_shard_rejects_topk_above_the_list(g4, torch_cuda):
    torch = torch_cuda
    s = g4.Sampler(0, 8, 262144)
    try:
        buf = torch.zeros(8 * 262144, device="cuda")
        lists = torch.zeros((8, g4.SHARD_LIST), dtype=torch.int64, device="cuda")
        counts = torch.zeros(8, dtype=torch.int32, device="cuda")
        rc = s.shard_lists(buf.data_ptr(), F32, 8, 131072, 262144, 0, 262144, g4.make_params(1.0, 300, 0.9), CAP,
                           lists.data_ptr(), counts.data_ptr(), check=False)
        assert rc == g4.ERR_ARG and "full-vocabulary rows" in s.last_error()
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


def test_nccl_one_rank_packed_exchange(g4, torch_cuda, tmp_path):
    # the NCCL form on a one-rank communicator (one GPU is enough): its
    # exchange packs each row's own slots; mixed top-K and full rows, per-row
    # params, must equal g4s_sample on the whole rows
    torch = torch_cuda
    import torch.multiprocessing as mp

    V, rows = 262144, 24
    x = synth.c5_logits(rows, step=78)
    prm = _full_params(rows)
    u = synth.uniforms(rows, 0x78)
    uid_path = str(tmp_path / "uid.bin")
    open(uid_path, "wb").write(g4.shard_unique_id())
    out_path = str(tmp_path / "tok%d.npy")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_nccl_rank, args=(1, uid_path, x, prm, u, out_path), nprocs=1, join=True)
    got = np.load(out_path % 0)
    xd = torch.from_numpy(x).cuda()
    ud = torch.from_numpy(u).cuda()
    want, _ = _unsharded(g4, torch, xd, F32, rows, V, prm, ud)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("mixed", [False, True])
def test_nccl_ranks(g4, torch_cuda, oracle, tmp_path, mixed):
    # top-K rows, and (mixed) full-vocabulary rows with the resolve and the
    # all-reduce; W = every GPU of the box, up to 8
    torch = torch_cuda
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    V, rows = 262144, 16
    x = synth.c5_logits(rows, step=77)
    prm = _full_params(rows) if mixed else synth.c5_params(rows)
    u = synth.uniforms(rows, 0x77)
    uid_path = str(tmp_path / "uid.bin")
    open(uid_path + ".tmp", "wb").write(g4.shard_unique_id())
    os.rename(uid_path + ".tmp", uid_path)
    out_path = str(tmp_path / "tok%d.npy")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_nccl_rank, args=(world, uid_path, x, prm, u, out_path), nprocs=world, join=True)
    toks = [np.load(out_path % r) for r in range(world)]
    for t in toks[1:]:
        np.testing.assert_array_equal(t, toks[0])
    xd = torch.from_numpy(x).cuda()
    ud = torch.from_numpy(u).cuda()
    want, _ = _unsharded(g4, torch, xd, F32, rows, V, prm, ud)
    np.testing.assert_array_equal(toks[0], want)
    topk = np.array([0 < K < V for _, K, _ in prm])
    if topk.any():
        pick = np.flatnonzero(topk)
        check_topk_rows(oracle, x[pick], F32, [prm[i] for i in pick], CAP, u[pick], {"tokens": toks[0][pick]})
