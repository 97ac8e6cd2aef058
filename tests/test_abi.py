"""The C-ABI library: it loads, exports every symbol include/g4sampler.h
declares, and its host-side behaviour (argument checks, errors, records) works
without a GPU.  No kernel is launched here."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "g4sampler.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(g4s_[a-z_0-9]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(g4):
    lib = g4.load()
    syms = declared_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) <= set(g4.SIGNATURES), set(syms) - set(g4.SIGNATURES)


def test_version_and_defaults(g4):
    lib = g4.load()
    assert lib.g4s_version() == 2
    p = g4.Params()
    lib.g4s_params_defaults(ctypes.byref(p))
    # TSamplingParams.SetDefaults (src/Gemma4.Model.pas:346-352)
    assert (p.temperature, p.top_k, p.repetition_penalty) == (1.0, 64, 1.0)
    assert abs(p.top_p - 0.95) < 1e-7


def test_params_record_layout(g4):
    # 4 x 4-byte fields at offsets 0/4/8/12, like the Pascal record
    assert ctypes.sizeof(g4.Params) == 16
    assert [getattr(g4.Params, f).offset for f in ("temperature", "top_k", "top_p", "repetition_penalty")] == [0, 4, 8, 12]


def test_create_rejects_bad_arguments(g4):
    lib = g4.load()
    h = ctypes.c_void_p()
    assert lib.g4s_create(0, 0, 100, 0, ctypes.byref(h)) == g4.ERR_ARG
    assert b"max_rows" in lib.g4s_last_error(None)
    assert lib.g4s_create(0, 1, 0, 0, ctypes.byref(h)) == g4.ERR_ARG
    assert lib.g4s_create(0, 1, 100, 0, None) == g4.ERR_ARG
    assert lib.g4s_create(0, 1, 1 << 30, 0, ctypes.byref(h)) == g4.ERR_CAPACITY
    assert not h.value


def test_null_context_calls_fail_cleanly(g4):
    lib = g4.load()
    p = g4.make_params()
    rc = lib.g4s_sample(None, None, 0, 1, 10, 10, ctypes.byref(p), 0, 30.0, None, None, None)
    assert rc == g4.ERR_ARG
    assert lib.g4s_destroy(None) == g4.OK
    assert lib.g4s_last_error(None) is not None
    assert lib.g4s_workspace_bytes(None) == 0
    assert lib.g4s_set_wait_limit(None, 1) == g4.ERR_ARG


def test_create_without_gpu_reports_unavailable(g4):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = g4.load()
    h = ctypes.c_void_p()
    rc = lib.g4s_create(0, 8, 1000, 0, ctypes.byref(h))
    assert rc == g4.ERR_UNAVAILABLE
    assert b"no CUDA device" in lib.g4s_last_error(None)
    with pytest.raises(g4.G4SError):
        g4.Sampler(0, 8, 1000)


def test_pascal_unit_declares_every_symbol():
    # the binding a maintainer adds to the reference (not compiled here: no FPC)
    # names every entry point of the header, with the header's ABI version
    pas = open(os.path.join(ROOT, "gemma4.pas_b200", "pascal", "G4Sampler.pas")).read()
    for s in declared_symbols():
        assert re.search(r"(function|procedure)\s+" + s + r"\b", pas), s
    ver = re.search(r"#define G4S_ABI_VERSION (\d+)", open(HEADER).read()).group(1)
    assert re.search(r"G4S_ABI_VERSION\s*=\s*" + ver + r"\s*;", pas)
