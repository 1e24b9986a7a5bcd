"""The reference's compile pass and price model around this library's
operator.

`load_reference()` imports them from their unmodified install in
baseline/_ref (oracle/install_reference.py, run by the build wherever the
reference checkout is present) with the one-file swap applied
(vectra_swap_plugin: `vectra_kernels.custom_ops` is custom_ops.py here).
"""

import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.path.join(ROOT, 'baseline', '_ref')


def installed() -> bool:
    """Whether the build installed the reference into baseline/_ref."""
    return os.path.isfile(os.path.join(REF, 'INSTALL.json'))


def load_reference():
    """The reference's `backend` (vectra_compiler.backend), `model`
    (models.price_transformer.model) and `compile_entry`
    (models.export.compile_entry), with the swap applied. Raises
    ImportError when baseline/_ref is missing."""
    if not installed():
        raise ImportError('the reference is not installed in baseline/_ref '
                          '(python oracle/install_reference.py)')
    for path in (REF, HERE):
        if path not in sys.path:
            sys.path.insert(0, path)
    # pylint: disable=import-outside-toplevel,unused-import
    import vectra_swap_plugin  # noqa: F401  (binds the swap on import)
    from models.export import compile_entry
    from models.price_transformer import model
    from vectra_compiler import backend
    return types.SimpleNamespace(backend=backend, model=model,
                                 compile_entry=compile_entry)
