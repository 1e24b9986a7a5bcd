"""Shared pytest configuration.

Tests marked `gpu` need a CUDA device (a B200 on the GPU box); they are
skipped where torch sees none. Everything else runs on the CPU.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line(
        'markers', 'gpu: needs a CUDA GPU (runs on the B200 box)')
    config.addinivalue_line(
        'markers', 'slow: takes more than a few seconds')


def pytest_collection_modifyitems(config, items):
    del config
    gpu_items = [item for item in items if 'gpu' in item.keywords]
    if not gpu_items:
        return
    import torch  # pylint: disable=import-outside-toplevel
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason='needs a CUDA GPU')
    for item in gpu_items:
        item.add_marker(skip)
