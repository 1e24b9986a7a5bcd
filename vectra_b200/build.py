"""Builds the two shared libraries of vectra_b200, in-tree.

* libvectra_rbf.so: the CUDA kernels and the C ABI (include/vectra_rbf.h
  and include/vectra_scan.h),
  compiled by nvcc for sm_100a only. No torch dependency.
* _vectra_rbf_torch.so: the PyTorch binding that registers the CUDA kernel
  of vectra::rbf_attention; links libvectra_rbf.so through $ORIGIN.

    python vectra_b200/build.py [--force] [--verbose]

(run as a script: `python -m vectra_b200.build` would first import the
package, which loads the library being rebuilt and fails if it is stale).

Objects go to vectra_b200/_build/ and are rebuilt when a source or header is
newer. nvcc cross-compiles without a GPU, so this runs on any host with the
CUDA toolkit.
"""

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, 'csrc')
INCLUDE = os.path.join(ROOT, 'include')
BUILD = os.path.join(PKG, '_build')
LIB = os.path.join(PKG, 'libvectra_rbf.so')
TORCH_EXT = os.path.join(PKG, '_vectra_rbf_torch.so')

CU_SOURCES = ['capi.cu', 'rbf_generic.cu', 'rbf_decode.cu', 'rbf_tc.cu',
              'rbf_small.cu', 'rbf_small_tc.cu', 'tma_maps.cu', 'scan.cu']
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


def cuda_home() -> str:
    home = os.environ.get('CUDA_HOME') or os.environ.get('CUDA_PATH')
    if home and os.path.isdir(home):
        return home
    nvcc = shutil.which('nvcc')
    if nvcc:
        return os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))
    return '/usr/local/cuda'


def _nvcc() -> str:
    return os.path.join(cuda_home(), 'bin', 'nvcc')


def _nvcc_version() -> str:
    out = subprocess.run([_nvcc(), '--version'], capture_output=True,
                         text=True, check=True).stdout
    for token in out.replace(',', ' ').split():
        if token.startswith('V') and token[1:2].isdigit():
            return token[1:]
    return 'unknown'


def _headers():
    found = [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    found += [os.path.join(CSRC, f) for f in os.listdir(CSRC)
              if f.endswith(('.cuh', '.h'))]
    return found


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(' '.join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True, check=False)
    if proc.returncode != 0:
        raise RuntimeError(f'command failed ({proc.returncode}): '
                           f'{" ".join(cmd)}\n{proc.stdout}\n{proc.stderr}')
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout + proc.stderr, flush=True)
    return proc


def nvcc_flags():
    return ARCH + [
        '-O3', '-lineinfo', '-std=c++17', '--expt-relaxed-constexpr',
        '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden',
        '-I', INCLUDE,
        f'-DVECTRA_NVCC_VERSION="{_nvcc_version()}"',
    ]


def build_library(force=False, verbose=False, extra_flags=(), lib_path=LIB,
                  build_dir=BUILD):
    """Compiles the kernels and links libvectra_rbf.so (or `lib_path`,
    e.g. a variant built with extra -D flags into its own `build_dir`)."""
    os.makedirs(build_dir, exist_ok=True)
    headers = _headers()
    flags = nvcc_flags() + list(extra_flags)
    objects, jobs = [], []
    for src in CU_SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(build_dir, src.replace('.cu', '.o'))
        objects.append(obj)
        if force or _stale(obj, [path] + headers):
            jobs.append([_nvcc()] + flags + ['-c', path, '-o', obj])
    if jobs:
        with concurrent.futures.ThreadPoolExecutor(len(jobs)) as pool:
            list(pool.map(lambda c: _run(c, verbose), jobs))
    if force or jobs or _stale(lib_path, objects):
        _run([_nvcc()] + ARCH + ['-shared', '-cudart', 'shared', '-o',
                                 lib_path]
             + objects + ['-Xlinker', '-rpath,' +
                          os.path.join(cuda_home(), 'lib64')], verbose)
    return lib_path


def build_torch_extension(force=False, verbose=False):
    """Compiles the PyTorch binding against the installed torch: the
    operator's registration and CUDA launcher (torch_ext.cpp) and its CPU
    implementation (rbf_cpu.cpp, parallel over planes with ATen's OpenMP
    thread pool, so it is compiled with -fopenmp and linked against the
    libgomp that torch itself loads)."""
    import torch  # pylint: disable=import-outside-toplevel
    from torch.utils import cpp_extension  # pylint: disable=import-outside-toplevel

    src = os.path.join(CSRC, 'torch_ext.cpp')
    cpu_src = os.path.join(CSRC, 'rbf_cpu.cpp')
    if not (force or _stale(TORCH_EXT, [src, cpu_src, LIB] + _headers())):
        return TORCH_EXT
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)  # pylint: disable=protected-access
    includes = cpp_extension.include_paths(device_type='cuda')
    common = ['-fPIC', '-std=c++17', f'-D_GLIBCXX_USE_CXX11_ABI={abi}',
              '-DTORCH_API_INCLUDE_EXTENSION_H',
              '-DTORCH_EXTENSION_NAME=_vectra_rbf_torch', '-I', INCLUDE,
              '-I', os.path.join(cuda_home(), 'include')]
    for inc in includes:
        common += ['-isystem', inc]
    os.makedirs(BUILD, exist_ok=True)
    cpu_obj = os.path.join(BUILD, 'rbf_cpu.o')
    _run(['g++', '-c', '-O3', '-fopenmp'] + common + [cpu_src, '-o', cpu_obj],
         verbose)
    cmd = ['g++', '-shared', '-O2'] + common + [src, cpu_obj, '-o', TORCH_EXT,
                                                '-L', PKG, '-lvectra_rbf']
    for libdir in cpp_extension.library_paths(device_type='cuda'):
        cmd += ['-L', libdir]
    cmd += ['-lc10', '-lc10_cuda', '-ltorch', '-ltorch_cpu', '-ltorch_cuda',
            '-l:libgomp.so.1', '-Wl,-rpath,$ORIGIN']
    _run(cmd, verbose)
    return TORCH_EXT


def build(force=False, verbose=False):
    build_library(force=force, verbose=verbose)
    build_torch_extension(force=force, verbose=verbose)


def main(argv=None):
    parser = argparse.ArgumentParser()
    parser.add_argument('--force', action='store_true')
    parser.add_argument('--verbose', action='store_true')
    args = parser.parse_args(argv)
    build(force=args.force, verbose=args.verbose)
    print(f'built {LIB}\nbuilt {TORCH_EXT}')


if __name__ == '__main__':
    sys.exit(main())
