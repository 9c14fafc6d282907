"""Shared fixtures. GPU tests carry @pytest.mark.gpu and need a CUDA device."""

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture
def device():
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    return torch.device("cuda")


@pytest.fixture(scope="session")
def ref_ext():
    """The reference's own CUDA kernels, built from its sources into oracle/_ref."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    from oracle import build_ref

    if build_ref.built_path() is None:
        pytest.fail("reference kernels not built (python oracle/build_ref.py)")
    return build_ref.load()
