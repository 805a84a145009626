"""Shared pytest setup: the `gpu` marker, import paths, and the engine fixture.

`-m "not gpu"` tests need no GPU: the oracle against its pins and golden
vectors, the descriptor encoders, the C ABI exports, host logic and the
multi-rank (gloo) paths.  `-m gpu` tests call libb2g's kernels through the C ABI
on cuda:0 and compare them with the CPU oracle.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "microbench-blackwell_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def engine():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import b2g

    eng = b2g.Engine(0)
    yield eng
    eng.close()
