import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs 2 or more CUDA devices")
    config.addinivalue_line("markers", "gpu_pending: needs a CUDA device; covers code that has not yet run on a GPU, "
                                       "so it is kept out of `-m gpu` until it has passed once (`-m gpu_pending`)")


def pytest_collection_modifyitems(config, items):
    import torch
    have = torch.cuda.is_available()
    ngpu = torch.cuda.device_count() if have else 0
    skip_gpu = pytest.mark.skip(reason="no CUDA device")
    skip_multi = pytest.mark.skip(reason="fewer than 2 CUDA devices")
    for it in items:
        if ("gpu" in it.keywords or "gpu_pending" in it.keywords) and not have:
            it.add_marker(skip_gpu)
        if "multigpu" in it.keywords and ngpu < 2:
            it.add_marker(skip_multi)
