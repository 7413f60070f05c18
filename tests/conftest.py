"""Shared test set-up: the `gpu` marker, import paths, and device fixtures.

CPU tests (-m "not gpu") check the oracle against golden vectors, the host
logic and that libsam3cuda loads and exports its ABI. GPU tests (-m gpu) are
the parity tests proper: they call libsam3cuda through its C ABI and compare
with the CPU oracle on the same seeded inputs.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "metal-sam-ios-experiments_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def sam3():
    import sam3cuda
    return sam3cuda


def _make_ctx(sam3, **cfg):
    return sam3.Context(0, **cfg)


@pytest.fixture(scope="session")
def ctx(sam3):
    """Context with the small test encoder configuration (dim 256, 4 heads)."""
    c = _make_ctx(sam3, embed_dim=256, num_heads=4, mlp_hidden=512, num_blocks=2, patch=14,
                  image_size=112, prune_after_block=1, keep_tokens=32, max_batch=2)
    yield c
    c.close()


@pytest.fixture(scope="session")
def ctx_full(sam3):
    """Context with the benchmark configuration (1008^2, dim 1024, 16 heads)."""
    c = _make_ctx(sam3, max_batch=1)
    yield c
    c.close()
