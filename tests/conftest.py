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


def compile_pass_installed():
    """Whether the build installed the reference's compile pass and price
    model (unmodified) into baseline/_ref. When it did, the tests that use
    them run, and fail if they cannot load them."""
    from tests import reference_swap  # pylint: disable=import-outside-toplevel
    return reference_swap.installed()


@pytest.fixture(scope='session')
def reference():
    """The reference's compile pass (`backend`), price model (`model`) and
    export module (`compile_entry`) from baseline/_ref, with the module name
    its replacement imports to register the operator
    (compiler/vectra_compiler/replacement.py:38-39) bound to this library
    (the one-file swap of kernels/vectra_kernels/custom_ops.py,
    tests/reference_swap/custom_ops.py)."""
    if not compile_pass_installed():
        pytest.skip('the reference is not installed in baseline/_ref (no '
                    'reference checkout at build time)')
    from tests import reference_swap  # pylint: disable=import-outside-toplevel
    return reference_swap.load_reference()


@pytest.fixture(scope='module')
def backend(reference):  # pylint: disable=redefined-outer-name
    """The reference's `vectra_compiler.backend` (see `reference`)."""
    return reference.backend
