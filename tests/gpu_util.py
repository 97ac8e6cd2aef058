"""Helpers of the GPU parity tests: run the CUDA sampler through the C ABI on
numpy inputs and compare with the CPU oracle."""
from __future__ import annotations

import math

import numpy as np

F32, BF16 = 0, 1
PROB_TOL = 1e-6          # relative tolerance on probabilities
BOUNDARY = 1e-6          # draws this close to a CDF boundary may differ (counted)


def run_gpu(sampler, torch, logits, dtype, params, softcap, u, cand_stride=0, full_probs=False,
            row_stride=None, offset_elems=0):
    """Samples rows of `logits` ([rows, V] float32, or uint16 bf16 bits) on the GPU.

    params: one g4sampler.Params (broadcast) or a list of (T, K, P) / Params.
    row_stride / offset_elems: lay the rows out with a larger stride and/or a
    start offset (to exercise unaligned and strided inputs)."""
    import g4sampler as g4

    rows, V = logits.shape
    stride = row_stride or V
    host = np.zeros((rows * stride + offset_elems,), dtype=logits.dtype)
    view = host[offset_elems:].reshape(rows, stride)
    view[:, :V] = logits
    if logits.dtype == np.uint16:
        dev = torch.from_numpy(host.view(np.int16)).cuda()
    else:
        dev = torch.from_numpy(host).cuda()
    esize = 2 if logits.dtype == np.uint16 else 4
    ptr = dev.data_ptr() + offset_elems * esize
    du = torch.from_numpy(np.ascontiguousarray(u, dtype=np.float64)).cuda()
    out = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    tprob = torch.zeros(rows, dtype=torch.float32, device="cuda")
    flags = torch.zeros(rows, dtype=torch.int32, device="cuda")
    o = g4.Outputs()
    o.token_prob = tprob.data_ptr()
    o.row_flags = flags.data_ptr()
    cids = cprobs = fprobs = None
    if cand_stride:
        cids = torch.full((rows, cand_stride), -9, dtype=torch.int32, device="cuda")
        cprobs = torch.zeros((rows, cand_stride), dtype=torch.float32, device="cuda")
        o.cand_ids, o.cand_probs, o.cand_stride = cids.data_ptr(), cprobs.data_ptr(), cand_stride
    if full_probs:
        fprobs = torch.zeros((rows, V), dtype=torch.float32, device="cuda")
        o.full_probs = fprobs.data_ptr()
    torch.cuda.synchronize()
    sampler.sample(ptr, dtype, rows, V, stride, params, float(softcap), du.data_ptr(), out.data_ptr(),
                   outputs=o)
    torch.cuda.synchronize()
    res = {"tokens": out.cpu().numpy(), "token_prob": tprob.cpu().numpy(), "flags": flags.cpu().numpy()}
    if cand_stride:
        res["cand_ids"] = cids.cpu().numpy()
        res["cand_probs"] = cprobs.cpu().numpy()
    if full_probs:
        res["full_probs"] = fprobs.cpu().numpy()
    return res


def row_params(params, r):
    import g4sampler as g4

    if isinstance(params, g4.Params):
        return params.temperature, params.top_k, params.top_p
    p = params[r]
    if isinstance(p, g4.Params):
        return p.temperature, p.top_k, p.top_p
    return p


def check_topk_rows(oracle, logits, dtype, params, softcap, u, res):
    """Top-K rows: ids, probabilities and tokens bit-identical to the oracle's
    fp32 transcription with the lower-id tie rule.  Returns counters."""
    stats = {"rows": 0, "boundary": 0, "heap_tie_rows": 0, "fallback": 0}
    for r in range(logits.shape[0]):
        T, K, P = row_params(params, r)
        x = oracle.as_f32(logits[r], dtype)
        p = oracle.params(T, K, P)
        tok, tr, ids, probs = oracle.sample(x, p, softcap, u[r], oracle.VARIANT_F32, oracle.TIE_LOWER,
                                            want_probs=True)
        heap_ids = oracle.topk(x, K, oracle.TIE_HEAP)
        if not np.array_equal(np.sort(heap_ids), ids):
            stats["heap_tie_rows"] += 1
        stats["rows"] += 1
        n = len(ids)
        if "cand_ids" in res:
            w = min(n, res["cand_ids"].shape[1])
            np.testing.assert_array_equal(res["cand_ids"][r, :w], ids[:w], err_msg=f"row {r} ids")
            assert (res["cand_ids"][r, w:] == -1).all()
            # probabilities: tolerance 1e-6 relative; the arithmetic is the same
            # fp32 sequence, so they are expected (and asserted) bit-identical
            np.testing.assert_array_equal(res["cand_probs"][r, :w], probs[:w], err_msg=f"row {r} probs")
        if tr["fallback"]:
            stats["fallback"] += 1
        if res["tokens"][r] != tok:
            assert tr["boundary"] < BOUNDARY, (r, res["tokens"][r], tok, tr)
            stats["boundary"] += 1
        else:
            if tok >= 0 and n and "token_prob" in res:
                # NaN probabilities (softcap disabled with +inf logits) compare equal
                want = probs[list(ids).index(tok)]
                assert np.array_equal(res["token_prob"][r], want, equal_nan=True), (r, res["token_prob"][r], want)
    return stats


def check_full_rows(oracle, logits, dtype, params, softcap, u, res, check_probs=True):
    """Full-vocabulary rows: tokens equal to the fp64 restatement except draws
    within 1e-6 of a CDF boundary (counted); every probability within
    1e-6 + 2^-23 * |s - M| relative of the fp64 probabilities (the reference
    rounds s - M to fp32 before Exp, src/Gemma4.Tensors.pas:659, so its own
    probabilities carry ~2^-24 * |s - M| relative error).  Also counts rows
    where the reference's fp32 transcription disagrees with fp64 (its drift)."""
    stats = {"rows": 0, "boundary": 0, "f32_vs_f64": 0, "max_rel_err": 0.0, "fallback": 0}
    for r in range(logits.shape[0]):
        T, K, P = row_params(params, r)
        x = oracle.as_f32(logits[r], dtype)
        p = oracle.params(T, K, P)
        t64, tr64, _, p64 = oracle.sample(x, p, softcap, u[r], oracle.VARIANT_F64, oracle.TIE_LOWER,
                                          want_probs=check_probs)
        t32, tr32, _, _ = oracle.sample(x, p, softcap, u[r], oracle.VARIANT_F32, oracle.TIE_LOWER)
        stats["rows"] += 1
        if t32 != t64:
            stats["f32_vs_f64"] += 1
        if tr64["fallback"]:
            stats["fallback"] += 1
        g = res["tokens"][r]
        if g != t64:
            assert tr64["boundary"] < BOUNDARY, (r, g, t64, tr64)
            stats["boundary"] += 1
        if check_probs and T > 0:
            gp = res["full_probs"][r].astype(np.float64)
            pmax = p64.max()
            live = p64 > 1e-30
            d = np.log(pmax / p64[live])
            tol = PROB_TOL + 2.0 ** -23 * d
            rel = np.abs(gp[live] - p64[live]) / p64[live]
            bad = rel > tol
            assert not bad.any(), (r, int(np.argmax(rel - tol)), float(rel.max()))
            stats["max_rel_err"] = max(stats["max_rel_err"], float(rel[d < 1].max(initial=0.0)))
            if g == t64 and g >= 0:
                tp = p64[g]
                assert abs(res["token_prob"][r] - tp) <= (PROB_TOL + 2.0 ** -23 * math.log(pmax / tp)) * tp
    return stats
