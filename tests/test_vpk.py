"""The weight archive through the C ABI (g4s_vpk_*): the reference's VPK
container (StdApp's TVFS) and TWeightStore's manifest, read on the host; the
LM head moved to the device and sampled on the GPU."""
import json
import os

import numpy as np
import pytest

import synth
from vpk_util import model_archive, pack


def _write(tmp_path, data, name="model.vpk"):
    p = os.path.join(str(tmp_path), name)
    with open(p, "wb") as f:
        f.write(data)
    return p


def test_open_find_and_read(g4, tmp_path):
    rng = np.random.default_rng(5)
    norm = rng.standard_normal(256).astype(np.float32)
    _, blocks = synth.c4_inputs(1, 256, 40, seed=9)
    path = _write(tmp_path, model_archive([
        ("model.language_model.norm.weight", "F32", norm.view(np.uint8), [256]),
        ("model.language_model.embed_tokens.weight", "Q4_0", blocks, [40, 256]),
    ]))
    with g4.Vpk(path) as v:
        assert len(v) == 2
        ti = v.find("model.language_model.embed_tokens.weight")
        assert ti.output_dtype == g4.DT_Q4_0 and ti.source_dtype == g4.DT_BF16
        assert ti.dims == (40, 256) and ti.size == 40 * 8 * 18 and ti.offset % 16 == 0
        raw, _ = v.tensor("model.language_model.embed_tokens.weight")
        np.testing.assert_array_equal(raw, blocks)
        raw, ti = v.tensor("model.language_model.norm.weight")
        assert ti.output_dtype == g4.DT_F32
        np.testing.assert_array_equal(raw.view(np.float32), norm)
        assert v.verify("E4B/manifest.json") == g4.OK
        assert v.verify("e4b\\WEIGHTS.bin") == g4.OK  # looked up normalised, as TVFS does
        with pytest.raises(g4.G4SError):
            v.find("no.such.tensor")


def test_rejects_bad_archives(g4, tmp_path):
    lib = g4.load()
    good = model_archive([("t", "F32", np.zeros(4, np.float32).view(np.uint8), [4])])
    cases = {
        "magic": pack({"E4B/manifest.json": b"{}"}, magic=b"ZIP0"),
        "version": pack({"E4B/manifest.json": b"{}"}, version=2),
        "truncated": good[:100],
        "no_manifest": pack({"E4B/weights.bin": b"\0" * 16}),
        "bad_json": pack({"E4B/manifest.json": b'{"tensors": [', "E4B/weights.bin": b""}),
        "no_tensors": pack({"E4B/manifest.json": b'{"other": 1}', "E4B/weights.bin": b""}),
        "outside": pack({"E4B/manifest.json": json.dumps({"tensors": [{"name": "t", "output_dtype": "F32",
                                                                        "offset": 8, "size": 16,
                                                                        "shape": [4]}]}).encode(),
                         "E4B/weights.bin": b"\0" * 16}),
    }
    for name, data in cases.items():
        p = _write(tmp_path, data, name + ".vpk")
        with pytest.raises(g4.G4SError) as e:
            g4.Vpk(p)
        assert e.value.code == g4.ERR_ARG, name
        assert lib.g4s_last_error(None), name
    with pytest.raises(g4.G4SError):
        g4.Vpk(os.path.join(str(tmp_path), "missing.vpk"))


def test_checksum_mismatch_is_reported(g4, tmp_path):
    data = bytearray(model_archive([("t", "F32", np.arange(8, dtype=np.float32).view(np.uint8), [8])]))
    data[-1] ^= 0x55  # a byte of weights.bin
    with g4.Vpk(_write(tmp_path, bytes(data))) as v:
        assert v.verify("E4B/weights.bin") == g4.ERR_STATE
        assert v.verify("E4B/manifest.json") == g4.OK


def test_custom_entry_paths(g4, tmp_path):
    arch = model_archive([("x", "F32", np.ones(4, np.float32).view(np.uint8), [4])], root="embeddings")
    p = _write(tmp_path, arch)
    with pytest.raises(g4.G4SError):
        g4.Vpk(p)  # the default E4B paths are absent
    with g4.Vpk(p, "embeddings/manifest.json", "embeddings/weights.bin") as v:
        assert v.find("x").dims == (4,)


@pytest.mark.gpu
def test_lmhead_from_archive_samples_like_direct_blocks(g4, torch_cuda, oracle, tmp_path):
    # the tied embed_tokens of an archive as the LM head: the same tokens as
    # the blocks handed to g4s_q4_repack directly
    torch = torch_cuda
    rows, hidden, vocab = 16, 2560, 8192
    h, blocks = synth.c4_inputs(rows, hidden, vocab, seed=33)
    path = _write(tmp_path, model_archive([("model.language_model.embed_tokens.weight", "Q4_0", blocks,
                                            [vocab, hidden])]))
    nib = torch.empty(vocab * hidden // 2, dtype=torch.uint8, device="cuda")
    sc = torch.empty(vocab * hidden // 32, dtype=torch.int16, device="cuda")
    with g4.Vpk(path) as v:
        assert v.load_lmhead(0, nib.data_ptr(), sc.data_ptr(), vocab) == (vocab, hidden)
        with pytest.raises(g4.G4SError):
            v.load_lmhead(0, nib.data_ptr(), sc.data_ptr(), vocab - 8)  # above max_vocab
    bd = torch.from_numpy(blocks).cuda()
    nib2 = torch.empty_like(nib)
    sc2 = torch.empty_like(sc)
    g4.q4_repack(bd.data_ptr(), vocab, hidden, nib2.data_ptr(), sc2.data_ptr())
    torch.cuda.synchronize()
    assert torch.equal(nib, nib2) and torch.equal(sc, sc2)
    hd = torch.from_numpy(h).cuda()
    u = torch.from_numpy(synth.uniforms(rows, 0x5A)).cuda()
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    with g4.Sampler(0, 64, vocab) as s:
        s.lmhead_sample(hd.data_ptr(), rows, hidden, nib.data_ptr(), sc.data_ptr(), vocab, g4.make_params(1.0, 64, 0.95),
                        30.0, u.data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
    assert (out.cpu().numpy() >= 0).all()
