"""Test configuration: registers the ``gpu`` marker (tests that need a B200)
and puts the repository root on ``sys.path`` so that ``oracle`` and the
``triton_flash_attention_b200`` loader module import."""

import contextlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a (B200) GPU")


@contextlib.contextmanager
def _deterministic_algorithms():
    import torch

    prev = torch.are_deterministic_algorithms_enabled()
    torch.use_deterministic_algorithms(True)
    try:
        yield
    finally:
        torch.use_deterministic_algorithms(prev)


@pytest.fixture
def deterministic():
    """Runs the test under ``torch.use_deterministic_algorithms(True)``: the
    backward then takes the separate dQ and dK/dV kernels, whose gradients
    are bitwise reproducible."""
    with _deterministic_algorithms():
        yield
