"""Test configuration: the ``gpu`` marker (tests that need a B200), import paths, and the CPU checkers' build."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
for path in (REPO, REPO / 'fused-zipnerf_b200', REPO / 'tests'):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200, sm_100a)')


@pytest.fixture(scope='session')
def oracle():
    from oracle.zf_oracle import Oracle, build
    build()
    return Oracle()


@pytest.fixture(scope='session')
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail('the gpu tests need a CUDA device')
    return torch.device('cuda:0')
