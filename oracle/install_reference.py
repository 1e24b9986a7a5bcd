"""Installs the reference's Python code that the compiled-model checks and
benchmark run, unchanged, into baseline/_ref (git-ignored; it travels to
the GPU box with the built libraries).

    python oracle/install_reference.py [REFERENCE_DIR]

What lands in baseline/_ref:

* the reference's two installable packages, `vectra_kernels` and
  `vectra_compiler` (pyproject.toml:61-63), by `pip install --no-index
  --no-build-isolation --no-deps --target` from a scratch copy of the
  checkout (the build writes into its source tree, and the checkout is
  read-only);
* the price-model application the packages do not include
  (pyproject.toml:59-60: `models/` runs from the repository root):
  `models/price_transformer` (the model, its encoders and its RBF
  attention), `models/export` (`compile_model`, `max_abs_error`,
  `ServingModel`) and `models/training/checkpoint.py`, which
  `compile_entry` imports — copied file for file, unmodified;
* the reference's own CPU test suites for the operator and the compile pass
  (`kernels/tests`, `compiler/tests`, with the repository-wide
  `conftest.py` and the `__init__.py` files that name their modules), under
  `ref_tests/`, unmodified, so that they can be run against this library's
  operator;
* INSTALL.json: the checkout it came from and the sha256 of every file.

Nothing here is imported by the library. tests/ load it (the compile pass
and the model around this library's operator, the reference's suites) and
so does bench.py's compiled-model mode (the reference's price model is the
workload; the operator inside it is this library's).

The checkout is found as REFERENCE_DIR, else $VECTRA_REFERENCE, else a
`reference` directory beside this repository. Exits 0 without installing
when there is none (a GPU box that only receives the installed copy).
"""

import hashlib
import json
import os
import shutil
import subprocess
import sys
import tempfile
import time

ORACLE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(ORACLE)
TARGET = os.path.join(ROOT, 'baseline', '_ref')
MARKER = os.path.join(TARGET, 'INSTALL.json')

# Files of the reference's price-model application, copied unchanged.
MODEL_FILES = (
    'models/__init__.py',
    'models/price_transformer/__init__.py',
    'models/price_transformer/candidate_encoder.py',
    'models/price_transformer/microhood.py',
    'models/price_transformer/model.py',
    'models/price_transformer/spatial_attention.py',
    'models/export/__init__.py',
    'models/export/compile_entry.py',
    'models/training/__init__.py',
    'models/training/checkpoint.py',
)
# The reference's test suites for the operator and the compile pass.
TEST_DIRS = ('kernels/tests', 'compiler/tests')
# Around the suites: the repository-wide conftest (the $CXX check and the
# gpu-marker skip) and the package files that name the suites' modules
# kernels.tests.* and compiler.tests.*.
SUITE_FILES = ('conftest.py', 'kernels/__init__.py', 'compiler/__init__.py')
# What pip needs from the checkout to build the two packages.
PACKAGING = ('pyproject.toml', 'README.md', 'LICENSE', 'NOTICE')
PACKAGE_DIRS = ('kernels', 'compiler')


def find_reference(argv):
    """The reference checkout's directory, or None."""
    for cand in (argv[1] if len(argv) > 1 else None,
                 os.environ.get('VECTRA_REFERENCE'),
                 os.path.join(os.path.dirname(ROOT), 'reference')):
        if cand and os.path.isfile(os.path.join(
                cand, 'compiler', 'vectra_compiler', 'backend.py')):
            return os.path.abspath(cand)
    return None


def _sha256(path):
    h = hashlib.sha256()
    with open(path, 'rb') as f:
        h.update(f.read())
    return h.hexdigest()


def _sources(ref):
    """Every file the install takes from the checkout (relative paths)."""
    files = list(MODEL_FILES)
    for top in PACKAGE_DIRS:
        pkg = os.path.join(ref, top)
        for name in os.listdir(pkg):
            if name.startswith('vectra_'):
                for f in sorted(os.listdir(os.path.join(pkg, name))):
                    if f.endswith('.py'):
                        files.append(f'{top}/{name}/{f}')
    for d in TEST_DIRS:
        for f in sorted(os.listdir(os.path.join(ref, d))):
            if f.endswith('.py'):
                files.append(f'{d}/{f}')
    return files + list(SUITE_FILES)


def up_to_date(ref):
    """Whether baseline/_ref already holds these sources, unchanged."""
    try:
        with open(MARKER, encoding='utf-8') as f:
            marker = json.load(f)
    except (OSError, ValueError):
        return False
    files = marker.get('files', {})
    return all(files.get(rel) == _sha256(os.path.join(ref, rel))
               for rel in _sources(ref))


def install(ref):
    if os.path.isdir(TARGET):
        shutil.rmtree(TARGET)
    os.makedirs(TARGET)
    with tempfile.TemporaryDirectory(prefix='vectra_ref_') as tmp:
        src = os.path.join(tmp, 'src')
        os.makedirs(src)
        for f in PACKAGING:
            if os.path.exists(os.path.join(ref, f)):
                shutil.copy2(os.path.join(ref, f), os.path.join(src, f))
        for d in PACKAGE_DIRS:
            shutil.copytree(os.path.join(ref, d), os.path.join(src, d),
                            ignore=shutil.ignore_patterns('__pycache__'))
        subprocess.run(
            [sys.executable, '-m', 'pip', 'install', '--quiet', '--no-index',
             '--no-build-isolation', '--no-deps', '--no-compile',
             '--target', TARGET, src], check=True, cwd=tmp)
    for rel in MODEL_FILES:
        dst = os.path.join(TARGET, rel)
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        shutil.copy2(os.path.join(ref, rel), dst)
    for d in TEST_DIRS:
        dst = os.path.join(TARGET, 'ref_tests', d)
        shutil.copytree(os.path.join(ref, d), dst,
                        ignore=shutil.ignore_patterns('__pycache__'))
    for rel in SUITE_FILES:
        shutil.copy2(os.path.join(ref, rel),
                     os.path.join(TARGET, 'ref_tests', rel))
    files = {rel: _sha256(os.path.join(ref, rel)) for rel in _sources(ref)}
    with open(MARKER, 'w', encoding='utf-8') as f:
        json.dump({'source': ref, 'installed_at': time.time(),
                   'files': files}, f, indent=1, sort_keys=True)
        f.write('\n')


def main(argv):
    ref = find_reference(argv)
    if ref is None:
        print('install_reference: no reference checkout found; '
              'baseline/_ref left as it is', file=sys.stderr)
        return 0
    if up_to_date(ref):
        return 0
    install(ref)
    print(f'install_reference: installed the reference compile pass and '
          f'price model from {ref} into {TARGET}', file=sys.stderr)
    return 0


if __name__ == '__main__':
    sys.exit(main(sys.argv))
