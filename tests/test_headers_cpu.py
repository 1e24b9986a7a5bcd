"""The C ABI headers compile on their own as C99 (pedantic, warnings as
errors) and as C++17: a cgo, JNI or plain C host includes them directly."""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, 'include')
HEADERS = sorted(h for h in os.listdir(INCLUDE) if h.endswith('.h'))


@pytest.mark.parametrize('header', HEADERS)
@pytest.mark.parametrize('compiler,flags,suffix', [
    ('gcc', ['-std=c99', '-pedantic'], '.c'),
    ('g++', ['-std=c++17'], '.cc')])
def test_header_compiles_alone(tmp_path, header, compiler, flags, suffix):
    if shutil.which(compiler) is None:
        pytest.skip(f'{compiler} not installed')
    src = tmp_path / f'use{suffix}'
    src.write_text(f'#include "{header}"\nint main(void) {{ return 0; }}\n')
    subprocess.run([compiler, *flags, '-Wall', '-Wextra', '-Werror',
                    '-I', INCLUDE, '-fsyntax-only', str(src)], check=True)
