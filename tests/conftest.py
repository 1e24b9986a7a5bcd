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


REF = os.path.join(ROOT, 'baseline', '_ref')


def compile_pass_installed():
    """Whether the reference's compile pass (installed unmodified into
    baseline/_ref) is here."""
    return os.path.isdir(os.path.join(REF, 'vectra_compiler'))


@pytest.fixture(scope='module')
def backend():
    """The reference's `vectra_compiler.backend`, with the module name its
    replacement imports to register the operator
    (compiler/vectra_compiler/replacement.py:38-39) bound to
    `vectra_b200.custom_ops` (the one-file swap of
    kernels/vectra_kernels/custom_ops.py)."""
    if not compile_pass_installed():
        pytest.skip('the reference compile pass is not installed in '
                    'baseline/_ref')
    import types  # pylint: disable=import-outside-toplevel
    import vectra_b200  # pylint: disable=import-outside-toplevel,unused-import
    from vectra_b200 import custom_ops  # pylint: disable=import-outside-toplevel
    names = ('vectra_kernels', 'vectra_kernels.custom_ops')
    saved = {n: sys.modules.get(n) for n in names}
    pkg = types.ModuleType('vectra_kernels')
    pkg.__path__ = []
    pkg.custom_ops = custom_ops
    sys.modules['vectra_kernels'] = pkg
    sys.modules['vectra_kernels.custom_ops'] = custom_ops
    sys.path.insert(0, REF)
    try:
        from vectra_compiler import backend as b  # pylint: disable=import-outside-toplevel
        yield b
    finally:
        sys.path.remove(REF)
        for n, m in saved.items():
            if m is None:
                sys.modules.pop(n, None)
            else:
                sys.modules[n] = m
