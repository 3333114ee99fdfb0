import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (CUDA sm_100a) and the built libmmp_b200.so")
    config.addinivalue_line("markers", "run_last: collected after every other test, so that under -x a failure "
                                       "there cannot hide the results of the rest of the suite")


def pytest_collection_modifyitems(config, items):
    items.sort(key=lambda it: 1 if "run_last" in it.keywords else 0)  # stable: file order otherwise kept
    # GPU tests are skipped, not failed, where no GPU is visible (the CPU suite runs everything else).
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
