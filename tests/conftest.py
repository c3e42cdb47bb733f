import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a B200 (sm_100a) GPU')
    config.addinivalue_line('markers', 'slow: takes more than a few seconds')


def pytest_collection_modifyitems(config, items):
    # GPU tests need a GPU; without one they are skipped rather than failed when selected explicitly
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if not has_gpu:
        skip = pytest.mark.skip(reason='no CUDA device')
        for item in items:
            if 'gpu' in item.keywords:
                item.add_marker(skip)


@pytest.fixture(scope='session')
def cuda_ops():
    """The sm_100a op library, loaded (fails loudly if it is missing on a GPU box)."""
    from xtier_b200 import ops
    ops.load()
    return ops
