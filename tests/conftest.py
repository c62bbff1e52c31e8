"""Shared pytest setup.

``-m "not gpu"`` runs the oracle's known-answer tests, the golden fixtures and
the host-side logic; ``-m gpu`` runs the CUDA parity tests through the C ABI.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_PARENT = os.path.join(REPO, "win-directml-java_b200")
for p in (REPO, PKG_PARENT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")


@pytest.fixture(scope="session")
def ctx():
    import torch
    import b200attn
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    c = b200attn.Context(0)
    yield c
    c.close()
