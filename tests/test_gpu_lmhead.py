"""LM head + sampling (config C4) through the C ABI: Q4_0 weights in the
reference block format (TQ4Block, src/Gemma4.Types.pas:139-142), repacked on
the device, logits by the tcgen05 fp16 GEMM (dequantized weights in TMEM), then
the sampler.

Logits are checked against the fp64 matvec of the same quantized weights
(restating CpuMatVecQ4, src/Gemma4.Tensors.pas:546-590, in exact arithmetic)
with the bound of the kernel's arithmetic: hidden and each weight are rounded
to fp16 (relative 2^-11 each) and products are summed in fp32, so
|err| <= 2^-9 * sum_k |w_k x_k| + 1e-6.  Tokens must equal the oracle's top-K
DoSample applied to the kernel's own logits (that path is bit-exact)."""
import numpy as np
import pytest

import synth
from gpu_util import F32, check_topk_rows

pytestmark = pytest.mark.gpu
CAP = 30.0


def _dequant(blocks, vocab, hidden):
    b = blocks.reshape(vocab, hidden // 32, 18)
    sc = (b[:, :, 0].astype(np.uint16) | (b[:, :, 1].astype(np.uint16) << 8)).view(np.float16).astype(np.float64)
    nb = b[:, :, 2:]
    q = np.empty((vocab, hidden // 32, 32), dtype=np.float64)
    q[:, :, 0::2] = (nb & 0xF).astype(np.float64) - 8
    q[:, :, 1::2] = (nb >> 4).astype(np.float64) - 8
    return (q * sc[:, :, None]).reshape(vocab, hidden)


def _run(g4, torch, s, h, blocks, vocab, hidden, prm, u):
    rows = h.shape[0]
    bd = torch.from_numpy(blocks).cuda()
    nib = torch.empty(vocab * hidden // 2, dtype=torch.uint8, device="cuda")
    sc = torch.empty(vocab * hidden // 32, dtype=torch.int16, device="cuda")
    g4.q4_repack(bd.data_ptr(), vocab, hidden, nib.data_ptr(), sc.data_ptr())
    hd = torch.from_numpy(h).cuda()
    ud = torch.from_numpy(u).cuda()
    out = torch.full((rows,), -5, dtype=torch.int32, device="cuda")
    logits = torch.empty((rows, vocab), dtype=torch.float32, device="cuda")
    s.lmhead_sample(hd.data_ptr(), rows, hidden, nib.data_ptr(), sc.data_ptr(), vocab, prm, CAP, ud.data_ptr(),
                    out.data_ptr(), logits_ptr=logits.data_ptr())
    torch.cuda.synchronize()
    assert s.lib.g4s_device_status(s.h) == g4.OK, s.last_error()  # no bounded wait ran out
    return out.cpu().numpy(), logits.cpu().numpy()


@pytest.mark.parametrize("rows,vocab", [(64, 8192), (5, 4104), (1, 2048)])
def test_lmhead_logits_and_tokens(g4, torch_cuda, oracle, rows, vocab):
    hidden = 2560
    h, blocks = synth.c4_inputs(rows, hidden, vocab)
    prm = [(1.0, 64, 0.95), (0.7, 20, 0.9), (0.0, 64, 0.9)] * (rows // 3 + 1)
    prm = prm[:rows]
    u = synth.uniforms(rows, 0xC4)
    s = g4.Sampler(0, 64, 262144)
    try:
        tok, lg = _run(g4, torch_cuda, s, h, blocks, vocab, hidden, prm, u)
    finally:
        s.close()
    W = _dequant(blocks, vocab, hidden)
    want = h.astype(np.float64) @ W.T
    bound = 2.0 ** -9 * (np.abs(h.astype(np.float64)) @ np.abs(W).T) + 1e-6
    err = np.abs(lg - want)
    assert (err <= bound).all(), float((err / bound).max())
    # the oracle's serial fp32 CpuMatVecQ4 on a few rows, for the record
    ref32 = oracle.matvec_q4(blocks, h[0], vocab, hidden)
    assert np.abs(ref32 - want[0]).max() < 1e-3
    check_topk_rows(oracle, lg, F32, prm, CAP, u, {"tokens": tok})


def test_lmhead_full_size_sample(g4, torch_cuda, oracle):
    # config C4 shapes: 64 x 2560 hidden, 262144 x 2560 Q4_0 weights (377 MB)
    rows, hidden, vocab = 64, 2560, 262144
    h, blocks = synth.c4_inputs(rows, hidden, vocab)
    u = synth.uniforms(rows, 0xC4, 1)
    prm = g4.make_params(1.0, 64, 0.95)
    s = g4.Sampler(0, 64, vocab)
    try:
        tok, lg = _run(g4, torch_cuda, s, h, blocks, vocab, hidden, prm, u)
    finally:
        s.close()
    pick = np.random.default_rng(4).choice(vocab, 3000, replace=False)
    W = _dequant(blocks.reshape(vocab, -1)[pick].reshape(-1), len(pick), hidden)
    want = h.astype(np.float64) @ W.T
    bound = 2.0 ** -9 * (np.abs(h.astype(np.float64)) @ np.abs(W).T) + 1e-6
    assert (np.abs(lg[:, pick] - want) <= bound).all()
    check_topk_rows(oracle, lg[::8], F32, prm, CAP, u[::8], {"tokens": tok[::8]})


def test_lmhead_with_fused_final_norm(g4, torch_cuda, oracle):
    # raw hidden states + the final RMSNorm weight: the prologue applies
    # CpuRmsNorm before the fp16 conversion
    torch = torch_cuda
    rows, hidden, vocab = 12, 2560, 4096
    h, blocks = synth.c4_inputs(rows, hidden, vocab)
    rng = np.random.default_rng(21)
    h = (h * rng.uniform(0.5, 3.0, (rows, 1)) + 0.1).astype(np.float32)  # not normalized
    gamma = rng.uniform(0.5, 1.5, hidden).astype(np.float32)
    u = synth.uniforms(rows, 0x4E)
    prm = g4.make_params(0.8, 40, 0.9)
    bd = torch.from_numpy(blocks).cuda()
    nib = torch.empty(vocab * hidden // 2, dtype=torch.uint8, device="cuda")
    sc = torch.empty(vocab * hidden // 32, dtype=torch.int16, device="cuda")
    g4.q4_repack(bd.data_ptr(), vocab, hidden, nib.data_ptr(), sc.data_ptr())
    hd, gd, ud = (torch.from_numpy(a).cuda() for a in (h, gamma, u))
    out = torch.full((rows,), -5, dtype=torch.int32, device="cuda")
    logits = torch.empty((rows, vocab), dtype=torch.float32, device="cuda")
    s = g4.Sampler(0, 64, vocab)
    try:
        s.lmhead_sample(hd.data_ptr(), rows, hidden, nib.data_ptr(), sc.data_ptr(), vocab, prm, CAP, ud.data_ptr(),
                        out.data_ptr(), logits_ptr=logits.data_ptr(), norm_ptr=gd.data_ptr(), norm_eps=1e-6)
        torch.cuda.synchronize()
        assert s.lib.g4s_device_status(s.h) == g4.OK, s.last_error()
    finally:
        s.close()
    lg, tok = logits.cpu().numpy(), out.cpu().numpy()
    xn = np.stack([oracle.rmsnorm(h[r], gamma, 1e-6) for r in range(rows)]).astype(np.float64)
    W = _dequant(blocks, vocab, hidden)
    want = xn @ W.T
    # fp32 norm differences (block vs serial sum of squares) are ~1e-7 relative,
    # far inside the fp16 bound
    bound = 2.0 ** -9 * (np.abs(xn) @ np.abs(W).T) + 1e-5
    assert (np.abs(lg - want) <= bound).all()
    check_topk_rows(oracle, lg, F32, prm, CAP, u, {"tokens": tok})


def test_lmhead_agreement_with_reference_paths(g4, torch_cuda, oracle):
    # The same C4 inputs through the reference's own LM-head arithmetic -- the
    # serial fp32 CpuMatVecQ4 (src/Gemma4.Tensors.pas:546-590) and the Q8_1 +
    # DP4A shaders its GPU path uses (gemma4_quantize_q8.comp,
    # gemma4_matvec_q4q8.comp) -- then the oracle's DoSample on those logits.
    # The three arithmetics round differently (fp16 operands here, fp32 and
    # int8 activations there), so survivor sets and tokens are compared as
    # agreement counts; the fp32 path must agree on nearly every survivor.
    import os

    torch = torch_cuda
    rows, hidden, vocab = 64, 2560, 262144
    h, blocks = synth.c4_inputs(rows, hidden, vocab)
    u = synth.uniforms(rows, 0xC4, 2)
    prm = g4.make_params(1.0, 64, 0.95)
    bd = torch.from_numpy(blocks).cuda()
    nib = torch.empty(vocab * hidden // 2, dtype=torch.uint8, device="cuda")
    sc = torch.empty(vocab * hidden // 32, dtype=torch.int16, device="cuda")
    g4.q4_repack(bd.data_ptr(), vocab, hidden, nib.data_ptr(), sc.data_ptr())
    hd, ud = torch.from_numpy(h).cuda(), torch.from_numpy(u).cuda()
    out = torch.full((rows,), -5, dtype=torch.int32, device="cuda")
    cid = torch.full((rows, 64), -9, dtype=torch.int32, device="cuda")
    o = g4.Outputs()
    o.cand_ids, o.cand_stride = cid.data_ptr(), 64
    s = g4.Sampler(0, 64, vocab)
    try:
        s.lmhead_sample(hd.data_ptr(), rows, hidden, nib.data_ptr(), sc.data_ptr(), vocab, prm, CAP, ud.data_ptr(),
                        out.data_ptr(), outputs=o)
        torch.cuda.synchronize()
    finally:
        s.close()
    tok, ids = out.cpu().numpy(), cid.cpu().numpy()
    nt = max(1, min(32, os.cpu_count() or 1))
    stats = {"rows": 0, "tok_f32": 0, "tok_q8": 0, "ids_f32": 0.0, "ids_q8": 0.0}
    for r in range(0, rows, 16):
        for name, lg in (("f32", oracle.matvec_q4_mt(blocks, h[r], vocab, hidden, nt)),
                         ("q8", oracle.matvec_q4q8(blocks, h[r], vocab, hidden, nt))):
            t, _, rid, _ = oracle.sample(lg, oracle.params(1.0, 64, 0.95), CAP, u[r], oracle.VARIANT_F32,
                                         oracle.TIE_LOWER)
            stats["tok_" + name] += int(t == tok[r])
            stats["ids_" + name] += len(set(rid.tolist()) & set(ids[r].tolist())) / 64.0
        stats["rows"] += 1
    print("C4 agreement with the reference's LM-head arithmetic:", stats)
    assert stats["ids_f32"] >= 0.95 * stats["rows"], stats
    assert stats["ids_q8"] >= 0.5 * stats["rows"], stats


# ---------------------------------------------------------------------------
# top-K selection in the LM head's epilogue (no logits output): the same
# tokens, probabilities and survivor lists as the unfused path, which writes
# the logits and samples them.
# ---------------------------------------------------------------------------
def _both_paths(g4, torch, h, blocks, vocab, hidden, prm, u, rows, kmax=256, with_outputs=True, norm=None):
    bd = torch.from_numpy(blocks).cuda()
    nib = torch.empty(vocab * hidden // 2, dtype=torch.uint8, device="cuda")
    sc = torch.empty(vocab * hidden // 32, dtype=torch.int16, device="cuda")
    g4.q4_repack(bd.data_ptr(), vocab, hidden, nib.data_ptr(), sc.data_ptr())
    hd = torch.from_numpy(h).cuda()
    ud = torch.from_numpy(u).cuda()
    nd = torch.from_numpy(norm).cuda() if norm is not None else None
    res = []
    s = g4.Sampler(0, 64, vocab)
    try:
        for mask in (0, g4.PHASE_LMHEAD_UNFUSED):
            out = torch.full((rows,), -5, dtype=torch.int32, device="cuda")
            tp = torch.full((rows,), -1.0, dtype=torch.float32, device="cuda")
            fl = torch.zeros(rows, dtype=torch.int32, device="cuda")
            ci = torch.full((rows, kmax), -7, dtype=torch.int32, device="cuda")
            cp = torch.full((rows, kmax), -7.0, dtype=torch.float32, device="cuda")
            o = g4.Outputs()
            o.phase_mask = mask
            if with_outputs:
                o.token_prob, o.row_flags = tp.data_ptr(), fl.data_ptr()
                o.cand_ids, o.cand_probs, o.cand_stride = ci.data_ptr(), cp.data_ptr(), kmax
            s.lmhead_sample(hd.data_ptr(), rows, hidden, nib.data_ptr(), sc.data_ptr(), vocab, prm, CAP,
                            ud.data_ptr(), out.data_ptr(), outputs=o, norm_ptr=nd.data_ptr() if nd is not None else 0)
            torch.cuda.synchronize()
            assert s.lib.g4s_device_status(s.h) == g4.OK, s.last_error()
            res.append({"tok": out.cpu().numpy(), "tp": tp.cpu().numpy(), "fl": fl.cpu().numpy(),
                        "ci": ci.cpu().numpy(), "cp": cp.cpu().numpy()})
    finally:
        s.close()
    return res


def _assert_same(a, b):
    for k in a:
        np.testing.assert_array_equal(a[k], b[k], err_msg=k)


def test_fused_epilogue_matches_unfused_c4(g4, torch_cuda):
    # config C4 (64 x 2560 hidden, 262144 x 2560 Q4_0) with per-row params:
    # K from 1 to 256, draws and greedy rows
    rows, hidden, vocab = 64, 2560, 262144
    h, blocks = synth.c4_inputs(rows, hidden, vocab)
    ks = [1, 2, 20, 40, 64, 100, 200, 256]
    prm = [(0.0 if r % 7 == 3 else 0.5 + 0.1 * (r % 9), ks[r % len(ks)], 0.5 + 0.5 * ((r * 37) % 100) / 100)
           for r in range(rows)]
    u = synth.uniforms(rows, 0xF4)
    fused, unfused = _both_paths(g4, torch_cuda, h, blocks, vocab, hidden, prm, u, rows)
    _assert_same(fused, unfused)
    assert (fused["tok"] >= 0).all()


def test_fused_epilogue_small_batches_and_norm(g4, torch_cuda):
    # fewer rows, a vocabulary just above the fused path's minimum (two waves
    # of 256-row tiles), broadcast params, the final RMSNorm in the prologue
    dev = torch_cuda.cuda.get_device_properties(0)
    vocab = 2 * dev.multi_processor_count * 256 + 8 * 37
    hidden = 1024
    for rows in (1, 7):
        h, blocks = synth.c4_inputs(rows, hidden, vocab, seed=rows)
        norm = (1.0 + 0.1 * np.random.default_rng(rows).standard_normal(hidden)).astype(np.float32)
        u = synth.uniforms(rows, 0xF5, rows)
        fused, unfused = _both_paths(g4, torch_cuda, h * 3.0, blocks, vocab, hidden, g4.make_params(0.8, 50, 0.9),
                                     u, rows, norm=norm)
        _assert_same(fused, unfused)


def _blocks_const(vocab, hidden, scale_bits, nibble):
    nblk = vocab * (hidden // 32)
    b = np.empty((nblk, 18), dtype=np.uint8)
    sb = np.broadcast_to(np.asarray(scale_bits, dtype=np.uint16).reshape(-1, 1), (vocab, hidden // 32)).reshape(-1)
    b[:, 0] = (sb & 0xFF).astype(np.uint8)
    b[:, 1] = (sb >> 8).astype(np.uint8)
    b[:, 2:] = np.uint8(nibble | (nibble << 4))
    return b.reshape(-1)


def test_fused_epilogue_heavy_ties(g4, torch_cuda):
    # every weight 0: every logit of every row equals 0, so the candidates are
    # the ids up to the threshold group's first id (more than the shared-memory
    # list for K = 200: the exact radix selection over global memory)
    rows, hidden, vocab = 4, 512, 131072
    blocks = _blocks_const(vocab, hidden, 0x3C00, 8)  # nibble 8 = value 0
    h = np.ones((rows, hidden), np.float32)
    prm = [(1.0, 200, 1.0), (0.0, 64, 0.9), (0.7, 256, 0.5), (1.0, 3, 1.0)]
    u = synth.uniforms(rows, 0xF6)
    fused, unfused = _both_paths(g4, torch_cuda, h, blocks, vocab, hidden, prm, u, rows)
    _assert_same(fused, unfused)
    for r, (_, K, _) in enumerate(prm):
        assert fused["tok"][r] < K  # ties: the K lowest ids survive
        np.testing.assert_array_equal(fused["ci"][r, :K], np.arange(K))


def test_fused_epilogue_logits_rising_with_id(g4, torch_cuda):
    # logit(v) grows with v: the sample (the lowest ids) gives a threshold that
    # nearly the whole rest of the vocabulary passes -- every row's candidate
    # list holds ~all ids (the exact radix path); tokens still equal
    rows, hidden, vocab = 3, 256, 131072
    sc = (np.linspace(0.001, 0.01, vocab).astype(np.float16)).view(np.uint16)
    blocks = _blocks_const(vocab, hidden, sc, 9)  # nibble 9 = value 1
    h = np.ones((rows, hidden), np.float32)
    prm = [(1.0, 64, 0.95), (0.0, 10, 0.9), (2.0, 256, 1.0)]
    u = synth.uniforms(rows, 0xF7)
    fused, unfused = _both_paths(g4, torch_cuda, h, blocks, vocab, hidden, prm, u, rows)
    _assert_same(fused, unfused)
    assert (fused["tok"] > vocab - 600).all()
