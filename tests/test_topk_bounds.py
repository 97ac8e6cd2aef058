"""CPU model of the bounds the top-K kernels prune with (csrc/g4s_topk.cu),
fuzzed over ties, masked logits (key 0) and sparse rows.  Each kernel keeps
only candidates at or above a bound computed from per-thread ("lane") maxima;
these tests restate those bounds in numpy and check the counting arguments
they rest on: no entry of the exact top K is ever pruned, and the kept sets
fit their buffers.  Keys are the kernels' order-preserving uint32 keys (0: not
a candidate); a composite key << 32 | ~id orders by value, then lower id."""
import numpy as np
import pytest

NTHREADS, NWARPS = 256, 8


def composites(keys, ids):
    return (keys.astype(np.uint64) << np.uint64(32)) | (~ids.astype(np.uint32)).astype(np.uint64)


def top_k(comp, keys, K):
    """The exact top K (largest composites among valid keys)."""
    c = np.sort(comp[keys > 0])[::-1]
    return set(c[:K].tolist())


def lane_maxima(keys_by_lane):
    return keys_by_lane.max(axis=1)


def kth_per_warp(lane_max, k):
    # each warp's k-th largest lane maximum (warp_sort_desc_u32, then lane k-1)
    return np.sort(lane_max.reshape(NWARPS, 32), axis=1)[:, ::-1][:, k - 1]


def random_keys(rng, n, kind):
    if kind == "normal":
        k = (rng.standard_normal(n) * 1000 + 2 ** 31).astype(np.uint32)
    elif kind == "ties":
        k = rng.integers(2 ** 31, 2 ** 31 + 3, n).astype(np.uint32)
    elif kind == "sparse":
        k = np.zeros(n, np.uint32)
        pick = rng.choice(n, max(1, n // 500), replace=False)
        k[pick] = rng.integers(1, 2 ** 32 - 1, pick.size).astype(np.uint32)
    else:  # masked mixture
        k = (rng.standard_normal(n) * 1000 + 2 ** 31).astype(np.uint32)
        k[rng.random(n) < 0.7] = 0
    return k


@pytest.mark.parametrize("kind", ["normal", "ties", "sparse", "masked"])
@pytest.mark.parametrize("K", [1, 7, 64, 256])
def test_stream_bound_cut_keeps_the_top_k(kind, K):
    # stream_bound_cut: entry i of the candidate buffer belongs to thread
    # i % 256; t = max(thr, min over warps of the warp's ceil(K/8)-th largest
    # lane maximum); the entries with key >= t survive.
    rng = np.random.default_rng(K * 31 + len(kind))
    for cnt in (257, 1000, 2100, 4096):
        keys = random_keys(rng, cnt, kind)
        ids = rng.permutation(10 ** 6)[:cnt].astype(np.uint32)
        comp = composites(keys, ids)
        per = -(-cnt // NTHREADS)
        pad = np.zeros(per * NTHREADS, np.uint32)
        pad[:cnt] = keys
        lane_max = pad.reshape(per, NTHREADS).max(axis=0)       # strided ownership
        t = int(kth_per_warp(lane_max, -(-K // NWARPS)).min())
        thr = 1
        t = max(t, thr)
        survivors = set(comp[keys >= t].tolist())
        assert top_k(comp, keys, K) <= survivors
        if (keys > 0).sum() >= K:
            assert len(survivors) >= K


@pytest.mark.parametrize("kind", ["normal", "ties", "sparse", "masked"])
@pytest.mark.parametrize("K", [1, 16, 64, 128])
def test_cluster_push_keeps_the_top_k(kind, K):
    # topk_cluster_kernel: 16 slices of 16384 ids, 64 per thread (element j of
    # thread t at j * 256 + t).  Each CTA publishes the ceil(K/16)-th largest of
    # its lane maxima and keeps a local bound (the smallest warp's ceil(K/8)-th
    # lane maximum); every CTA pushes its keys >= max(smallest published, local
    # bound), or, with more than 128 of them, the prefix of its exact top K.
    rng = np.random.default_rng(K * 7 + len(kind))
    C, S, EPT = 16, 16384, 64
    keys = random_keys(rng, C * S, kind)
    ids = np.arange(C * S, dtype=np.uint32)
    comp = composites(keys, ids)
    j0, kp = -(-K // C), -(-K // NWARPS)
    bound, tloc = [], []
    for r in range(C):
        sk = keys[r * S:(r + 1) * S].reshape(EPT, NTHREADS)     # [j][thread]
        lm = sk.max(axis=0)
        bound.append(int(np.sort(lm)[::-1][j0 - 1]))
        tloc.append(int(kth_per_warp(lm, kp).min()))
    T = min(bound)
    pushed = set()
    total = 0
    for r in range(C):
        thr = max(T, tloc[r], 1)
        sl = slice(r * S, (r + 1) * S)
        sel = keys[sl] >= thr
        if sel.sum() <= 128:
            got = comp[sl][sel]
        else:
            own = np.sort(comp[sl][keys[sl] > 0])[::-1][:K]
            got = own[own >= (np.uint64(thr) << np.uint64(32))]
        total += got.size
        pushed |= set(got.tolist())
    assert top_k(comp, keys, K) <= pushed
    assert total <= C * 128
