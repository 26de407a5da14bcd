"""Test configuration: the `gpu` marker and import paths.

CPU tests (`-m "not gpu"`) cover the oracle against the golden fixtures, the
host-side logic and the C-ABI library's exports. GPU tests (`-m gpu`) are the
parity tests proper: they call the sm_100a kernels through the C ABI and
compare against the oracle or a plain PyTorch fp32 reference.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "subnetwork-speculative-decoding_b200")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built kernel library")
    config.addinivalue_line("markers", "slow: long-running parity case")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
