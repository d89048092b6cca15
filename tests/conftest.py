"""Test configuration: the ``gpu`` marker selects tests that need a B200 (``pytest -m gpu``); everything else runs on
the CPU (``pytest -m "not gpu"``)."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / 'tests' / 'golden'


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200, sm_100a)')


@pytest.fixture(scope='session')
def golden():
    import torch

    def load(name):
        return torch.load(GOLDEN / name, weights_only=False)
    return load


@pytest.fixture(scope='session', autouse=True)
def _threads():
    import torch
    torch.set_num_threads(min(8, os.cpu_count() or 1))
