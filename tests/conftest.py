import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (CUDA sm_100a) and the built libmmp_b200.so")
    config.addinivalue_line("markers", "run_last(order=0): collected after every other test, so that under -x a "
                                       "failure there cannot hide the results of the rest of the suite; among "
                                       "them, higher orders run later")


def _run_last_key(it) -> tuple[int, int]:
    m = it.get_closest_marker("run_last")
    if m is None:
        return (0, 0)
    return (1, int(m.kwargs.get("order", m.args[0] if m.args else 0)))


def pytest_collection_modifyitems(config, items):
    items.sort(key=_run_last_key)  # stable: file order otherwise kept
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
