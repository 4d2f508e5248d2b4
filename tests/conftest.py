import os
import sys

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "multigpu: needs two or more B200 GPUs")


def pytest_collection_modifyitems(config, items):
    import torch

    have_gpu = torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    ngpu = torch.cuda.device_count() if have_gpu else 0
    skip_gpu = pytest.mark.skip(reason="no sm_100 GPU visible")
    skip_multi = pytest.mark.skip(reason="fewer than 2 GPUs visible")
    for item in items:
        if "gpu" in item.keywords and not have_gpu:
            item.add_marker(skip_gpu)
        if "multigpu" in item.keywords and ngpu < 2:
            item.add_marker(skip_multi)
