import pathlib
import sys

import pytest

REPO = pathlib.Path(__file__).resolve().parents[1]
for p in (REPO / 'dcss-auto_b200', REPO / 'oracle', REPO / 'tests'):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200); run with -m gpu')


@pytest.fixture(scope='session')
def oracle_lib():
    import oracle
    oracle.build()
    return oracle


def cuda_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
