"""Shared fixtures.  GPU tests are marked `gpu` and run only on a B200 box
(`pytest -m gpu`); everything else runs on the CPU (`pytest -m "not gpu"`)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gemma4.pas_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (CUDA) and the built libg4sampler.so")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.load()
    return O


@pytest.fixture(scope="session")
def g4():
    import g4sampler

    g4sampler.load()
    return g4sampler


@pytest.fixture(scope="session")
def torch_cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but torch.cuda is not available")
    return torch


@pytest.fixture(scope="session")
def sampler(g4, torch_cuda):
    torch_cuda.cuda.init()
    s = g4.Sampler(device=0, max_rows=1024, max_vocab=262144)
    yield s
    s.close()
