import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PACKAGE = ROOT / 'dynamic-kv-cache_b200'
GOLDEN = ROOT / 'tests' / 'golden'
for p in (str(ROOT), str(PACKAGE)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200, sm_100a)')


@pytest.fixture(scope='session')
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip('CUDA required')
    return torch.device('cuda', 0)
