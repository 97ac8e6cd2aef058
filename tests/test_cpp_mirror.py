"""The C++ host mirror (include/g4sampler.hpp: TSamplingParams / TSampler.DoSample)
compiled against the C ABI: error behaviour on the CPU, token parity on the GPU."""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gemma4.pas_b200")
SRC = os.path.join(ROOT, "tests", "cpp", "host_mirror.cpp")


@pytest.fixture(scope="module")
def exe(tmp_path_factory, g4):
    out = str(tmp_path_factory.mktemp("cpp") / "host_mirror")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), SRC, "-o", out,
                    "-L", PKG, "-lg4sampler", f"-Wl,-rpath,{PKG}"], check=True)
    return out


def test_mirror_errors_without_gpu(exe):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = subprocess.run([exe, "cpu"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "G4S8" in r.stdout  # G4S_ERR_UNAVAILABLE recorded in GetErrors()


@pytest.mark.gpu
def test_mirror_dosample_matches_oracle(exe, oracle, tmp_path):
    import synth

    for step, (T, K, P) in enumerate([(1.0, 64, 0.95), (0.7, 40, 0.9), (1.0, 0, 0.95), (0.0, 64, 0.9)]):
        x = synth.c1_logits(step)
        f = tmp_path / f"row{step}.f32"
        x.astype(np.float32).tofile(f)
        u = 0.123 + 0.2 * step
        r = subprocess.run([exe, "gpu", str(f), str(x.size), repr(u), repr(T), str(K), repr(P), "30"],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stdout + r.stderr
        got = int(r.stdout.split()[-1])
        variant = oracle.VARIANT_F64 if K <= 0 else oracle.VARIANT_F32
        want, tr, _, _ = oracle.sample(x, oracle.params(T, K, P), 30.0, u, variant, oracle.TIE_LOWER)
        assert got == want or tr["boundary"] < 1e-6, (step, got, want)
