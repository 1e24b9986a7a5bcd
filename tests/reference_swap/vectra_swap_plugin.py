"""The one-file swap, applied on import: the reference's
`vectra_kernels.custom_ops` becomes this directory's custom_ops.py (this
library's operator).

Loaded as a pytest plugin (`-p vectra_swap_plugin`, imported before any
conftest), it lets the reference's own suites run against this library:
every `from vectra_kernels import custom_ops` in them and in the compile
pass (compiler/vectra_compiler/replacement.py:38-39) then registers and
calls this library's operator. Needs the reference's `vectra_kernels`
package (installed unmodified in baseline/_ref) on the path.
"""

import importlib.util
import os
import sys

_HERE = os.path.dirname(os.path.abspath(__file__))


def bind():
    """Binds vectra_kernels.custom_ops to the swap file (idempotent)."""
    import vectra_kernels  # pylint: disable=import-outside-toplevel
    current = sys.modules.get('vectra_kernels.custom_ops')
    if current is not None and getattr(current, '__file__', '') == \
            os.path.join(_HERE, 'custom_ops.py'):
        return current
    spec = importlib.util.spec_from_file_location(
        'vectra_kernels.custom_ops', os.path.join(_HERE, 'custom_ops.py'))
    module = importlib.util.module_from_spec(spec)
    sys.modules['vectra_kernels.custom_ops'] = module
    spec.loader.exec_module(module)
    vectra_kernels.custom_ops = module
    return module


bind()
