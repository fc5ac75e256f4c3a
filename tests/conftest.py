"""Test configuration: registers the ``gpu`` marker (tests that need a B200)
and puts the repository root on ``sys.path`` so that ``oracle`` and the
``triton_flash_attention_b200`` loader module import."""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a (B200) GPU")
