"""Vocabulary-sharded mode on the CPU.

The partition and exact merge that g4s_shard_lists / g4s_shard_merge run on
the GPU, restated over the oracle and run as world_size-2 gloo ranks: each
rank takes its contiguous slice, keeps the slice's top K (lower-id ties), the
lists are all-gathered, and the merged top K must equal the whole row's top K,
so the sampled token equals unsharded DoSample's.  Plus the C-ABI argument
checks of the shard entry points (no GPU needed)."""
import ctypes
import datetime
import os
import socket

import numpy as np
import pytest

CAP = 30.0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, V, rows):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import g4sampler as g4
        import synth
        from oracle import oracle as O

        O.load()
        x = synth.c5_logits(rows, vocab=V, step=3)
        x[:, 100:140] = 1.5  # ties across the slice boundary region
        prm = synth.c5_params(rows)
        u = synth.uniforms(rows, 0x5A)
        lo, hi = g4.shard_slices(V, world)[rank]
        tokens = []
        for r in range(rows):
            T, K, P = prm[r]
            ids = O.topk(x[r, lo:hi], K) + lo  # the slice's top K, ascending ids
            lists = [None] * world
            dist.all_gather_object(lists, (x[r, ids].tolist(), ids.tolist()))
            cand = [(v, i) for vals, idl in lists for v, i in zip(vals, idl)]
            cand.sort(key=lambda c: (-c[0], c[1]))  # value descending, lower id first
            merged = np.array(sorted(i for _, i in cand[:K]), dtype=np.int64)
            np.testing.assert_array_equal(merged, O.topk(x[r], K), err_msg=f"row {r}")
            masked = np.full(V, -np.inf, dtype=np.float32)
            masked[merged] = x[r, merged]
            tok_shard = O.sample(masked, O.params(T, K, P), CAP, u[r])[0]
            tok_full = O.sample(x[r], O.params(T, K, P), CAP, u[r])[0]
            assert tok_shard == tok_full, (r, tok_shard, tok_full)
            tokens.append(tok_shard)
        # every rank drew the same tokens
        allt = [None] * world
        dist.all_gather_object(allt, tokens)
        assert all(t == allt[0] for t in allt)
    finally:
        dist.destroy_process_group()


def test_sharded_merge_is_exact_two_gloo_ranks():
    import torch.multiprocessing as mp

    mp.spawn(_rank_main, args=(2, _free_port(), 6000, 24), nprocs=2, join=True)


def _full_rank_main(rank, world, port, V, rows):
    """Full-vocabulary rows: each rank summarises its slice (first maximum and
    its id, fp64 mass), the summaries are all-gathered, every rank finds the
    slice whose share crosses fl32(u * top_p) * S, that rank walks its slice
    to the token, and a max all-reduce hands it to the others (-1 elsewhere).
    The token must be the unsharded fp64 restatement's."""
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import g4sampler as g4
        import synth
        from oracle import oracle as O

        O.load()
        x = synth.c5_logits(rows, vocab=V, step=5)
        x[1, V - 7] = 30.0  # the maximum in the last slice
        x[2, :] = 0.25      # every id tied: greedy takes id 0, draws land by u alone
        lo, hi = g4.shard_slices(V, world)[rank]
        for r in range(rows):
            T, P = (0.0, 0.9) if r % 4 == 3 else (0.6 + 0.1 * r, 0.8 + 0.01 * r)
            u = float(synth.uniforms(rows, 0xF0)[r])
            prm = O.params(T, 0, P)
            want, tr, _, probs = O.sample(x[r], prm, CAP, u, O.VARIANT_F64, O.TIE_LOWER, want_probs=True)
            # the slice summary
            xs = x[r, lo:hi]
            mloc = int(np.argmax(xs))  # first maximum of the slice (softcap and 1/T keep the order)
            z = float(probs[lo:hi].sum()) if T > 0 else 0.0
            allsum = [None] * world
            dist.all_gather_object(allsum, (float(xs[mloc]), lo + mloc, z))
            tok = torch.tensor([-1], dtype=torch.int64)
            if T <= 0:
                best = max(range(world), key=lambda w: (allsum[w][0], -allsum[w][1]))
                tok[0] = allsum[best][1]
            else:
                S = sum(a[2] for a in allsum)
                target = float(np.float32(u * np.float32(P))) * S
                cum, owner, t_loc = 0.0, -1, 0.0
                for w in range(world):
                    if allsum[w][2] > 0 and cum + allsum[w][2] >= target:
                        owner, t_loc = w, target - cum
                        break
                    cum += allsum[w][2]
                assert owner >= 0, r
                if owner == rank:
                    c = np.cumsum(probs[lo:hi])
                    tok[0] = lo + min(int(np.searchsorted(c, min(t_loc, c[-1]))), hi - lo - 1)
            dist.all_reduce(tok, op=dist.ReduceOp.MAX)
            if int(tok[0]) != want:
                assert tr["boundary"] < 1e-6, (r, int(tok[0]), want, tr)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_full_rows_gloo_ranks(world):
    import torch.multiprocessing as mp

    mp.spawn(_full_rank_main, args=(world, _free_port(), 5000, 12), nprocs=world, join=True)


def test_shard_slices_cover_the_vocabulary(g4):
    for V, W in ((262144, 8), (262144, 3), (1000, 7), (9, 2)):
        sl = g4.shard_slices(V, W)
        assert sl[0][0] == 0 and sl[-1][1] == V
        assert all(a[1] == b[0] for a, b in zip(sl, sl[1:]))


def test_shard_abi_rejects_bad_calls(g4):
    lib = g4.load()
    p = g4.make_params(1.0, 64, 0.95)
    bp = ctypes.byref(p)
    assert lib.g4s_shard_lists(None, None, 0, 1, 1000, 1000, 0, 1000, bp, 0, 30.0, None, None, None) == g4.ERR_ARG
    assert lib.g4s_shard_resolve(None, None, 0, 1, 1000, 1000, 0, 0, bp, 0, 30.0, None, None, None,
                                 None) == g4.ERR_ARG
    assert lib.g4s_shard_merge(None, None, None, 2, 1, 1000, bp, 0, 30.0, None, None, None, None) == g4.ERR_ARG
    assert lib.g4s_shard_init(None, 2, 0, 262144, None) == g4.ERR_ARG
    assert lib.g4s_shard_unique_id(None) == g4.ERR_ARG
    assert lib.g4s_shard_set_timeout(None, 1000) == g4.ERR_ARG
    assert lib.g4s_shard_wait(None, None, 1000) == g4.ERR_ARG
    assert lib.g4s_shard_abort(None) == g4.ERR_ARG
    assert lib.g4s_shard_sample(None, None, 0, 1, 1000, bp, 0, 30.0, None, None, None, None) == g4.ERR_ARG
    assert b"ctx is NULL" in lib.g4s_last_error(None)
