"""The C ABI of libvectra_rbf.so, on the CPU (no kernel is launched).

Checks that the library loads, that it exports every function
include/vectra_rbf.h declares, and that argument validation and kernel
selection (vectra_rbf_select_kernel, which never touches a device) follow
the reference's rules: rank-4 q/k/v of one dtype
(compiler/vectra_compiler/replacement.py:42,135-138), scale broadcast to
[B,H,1,1] (kernels/vectra_kernels/reference.py:41-43), key_bias
left-padded, constant across queries and broadcast to [B,1|H,1,Nk]
(kernels/vectra_kernels/spatial_rbf_attention.py:220-234).
"""

import ctypes
import os
import re

import pytest

from vectra_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, 'include', 'vectra_rbf.h')
FAKE = 0x10000  # a 16-byte aligned non-null address; never dereferenced


def _declared_functions():
    text = open(HEADER, encoding='utf-8').read()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    return sorted(set(re.findall(r'\b(vectra_rbf_\w+)\s*\(', text)))


def test_library_exports_every_declared_function():
    declared = _declared_functions()
    assert declared, 'no declarations parsed'
    assert sorted(_lib.EXPORTED) == declared
    for name in declared:
        assert hasattr(_lib.LIB, name), name


def test_status_strings():
    assert _lib.strerror(_lib.OK) == 'ok'
    assert _lib.strerror(_lib.ERR_BIAS_QUERY) == (
        'key_bias must be constant across queries')
    assert _lib.strerror(12345) == 'unknown status'
    assert [_lib.kernel_name(k) for k in range(8)] == [
        'none', 'generic', 'decode', 'tc', 'invalid', 'small', 'small_tc',
        'invalid']


def test_build_info_names_the_architecture():
    assert 'sm_100a' in _lib.build_info()


def _tensor(shape, dtype=_lib.BF16, strides=None, addr=FAKE):
    t = _lib.Tensor()
    t.data = addr
    t.dtype = dtype
    t.ndim = len(shape)
    if strides is None:
        strides, acc = [], 1
        for s in reversed(shape):
            strides.insert(0, acc)
            acc *= s
    for i, (s, st) in enumerate(zip(shape, strides)):
        t.size[i] = s
        t.stride[i] = st
    return t


def _args(B=4, H=8, nq=1, nk=64, d=64, dv=64, dtype=_lib.BF16,
          scale_shape=(1, 8, 1, 1), bias_shape=None, bias_dtype=_lib.BF16,
          q_strides=None, flags=0):
    a = _lib.Args()
    a.q = _tensor((B, H, nq, d), dtype, q_strides)
    a.k = _tensor((B, H, nk, d), dtype)
    a.v = _tensor((B, H, nk, dv), dtype)
    a.scale = _tensor(scale_shape, _lib.F32)
    if bias_shape is not None:
        a.key_bias = _tensor(bias_shape, bias_dtype)
    a.out = FAKE
    st = [H * nq * dv, nq * dv, dv, 1]
    for i in range(4):
        a.out_stride[i] = st[i]
    a.flags = flags
    return a


def _select(a):
    return _lib.LIB.vectra_rbf_select_kernel(ctypes.byref(a))


def test_serving_shape_selects_the_decode_kernel():
    assert _select(_args()) == _lib.KERNEL_DECODE
    assert _select(_args(bias_shape=(4, 1, 1, 64))) == _lib.KERNEL_DECODE
    assert _select(_args(d=128, dv=128)) == _lib.KERNEL_DECODE
    assert _select(_args(d=32, dv=32)) == _lib.KERNEL_DECODE
    # The retired flag bit (an mma.sync decode kernel), like any unknown
    # bit, is refused rather than ignored.
    assert _select(_args(flags=0x8)) == _lib.ERR_FORCED
    assert _select(_args(flags=0x100)) == _lib.ERR_FORCED


def test_config1_fp32_selects_decode():
    a = _args(B=8, H=4, nk=16, d=32, dv=32, dtype=_lib.F32,
              scale_shape=(1, 4, 1, 1))
    assert _select(a) == _lib.KERNEL_DECODE


def test_short_key_lists_select_the_small_kernels():
    # The compiled model's sites: [1024, 8, 65, 32] strided views, on the
    # mma.sync form; the tcgen05 form (Nq <= 96, Nk <= 128 - D) only when
    # forced.
    st = (65 * 768, 32, 768, 1)
    a = _args(B=1024, nq=65, nk=65, d=32, dv=32, bias_shape=(1024, 1, 1, 65),
              q_strides=st)
    a.k = _tensor((1024, 8, 65, 32), strides=st)
    a.v = _tensor((1024, 8, 65, 32), strides=st)
    assert _select(a) == _lib.KERNEL_SMALL
    a.flags = _lib.FLAG_FORCE_SMALL_TC
    assert _select(a) == _lib.KERNEL_SMALL_TC
    for nq, nk, d in ((96, 96, 32), (64, 64, 64)):
        assert _select(_args(nq=nq, nk=nk, d=d, dv=d)) == _lib.KERNEL_SMALL
        assert _select(_args(nq=nq, nk=nk, d=d, dv=d,
                             flags=_lib.FLAG_FORCE_SMALL_TC)) == (
                                 _lib.KERNEL_SMALL_TC)
    # More queries than three TMEM lane quarters, or keys past the slot's
    # S columns: not the tcgen05 form.
    for nq, nk, d in ((97, 65, 32), (65, 97, 32), (65, 65, 64)):
        assert _select(_args(nq=nq, nk=nk, d=d, dv=d)) == _lib.KERNEL_SMALL
        assert _select(_args(nq=nq, nk=nk, d=d, dv=d,
                             flags=_lib.FLAG_FORCE_SMALL_TC)) == (
                                 _lib.ERR_FORCED)
    assert _select(_args(nq=2, nk=128, d=64, dv=64)) == _lib.KERNEL_SMALL
    # fp32, more than 128 keys, or D outside {32, 64}: not this kernel.
    assert _select(_args(nq=65, nk=65, d=32, dv=32, dtype=_lib.F32)) == (
        _lib.KERNEL_GENERIC)
    assert _select(_args(nq=65, nk=129, d=32, dv=32)) == _lib.KERNEL_GENERIC
    assert _select(_args(nq=65, nk=65, d=128, dv=128)) == _lib.KERNEL_GENERIC
    # Row strides that are not 16-byte multiples rule out the TMA boxes.
    a = _args(nq=65, nk=65, d=32, dv=32, q_strides=(8 * 65 * 40, 65 * 40, 40,
                                                       1))
    assert _select(a) == _lib.KERNEL_SMALL
    a = _args(nq=65, nk=65, d=32, dv=32, q_strides=(8 * 65 * 36, 65 * 36, 36,
                                                       1))
    assert _select(a) == _lib.KERNEL_GENERIC
    assert _select(_args(nq=65, nk=65, d=32, dv=32,
                         flags=_lib.FLAG_FORCE_SMALL)) == _lib.KERNEL_SMALL
    assert _select(_args(flags=_lib.FLAG_FORCE_SMALL)) == _lib.ERR_FORCED


def test_self_attention_and_odd_widths_fall_to_generic():
    assert _select(_args(nq=65, nk=65, d=48, dv=48)) == _lib.KERNEL_GENERIC
    assert _select(_args(d=100, dv=128)) == _lib.KERNEL_GENERIC
    assert _select(_args(d=64, dv=32)) == _lib.KERNEL_GENERIC


def test_non_unit_inner_stride_falls_to_generic():
    a = _args(q_strides=(8 * 64 * 2, 64 * 2, 64 * 2, 2))
    assert _select(a) == _lib.KERNEL_GENERIC


def test_forced_kernels():
    assert _select(_args(flags=_lib.FLAG_FORCE_GENERIC)) == (
        _lib.KERNEL_GENERIC)
    assert _select(_args(nq=2, flags=_lib.FLAG_FORCE_DECODE)) == (
        _lib.ERR_FORCED)


def test_empty_problems_launch_nothing():
    assert _select(_args(B=0)) == _lib.KERNEL_NONE
    assert _select(_args(nq=0)) == _lib.KERNEL_NONE


@pytest.mark.parametrize('shape,status', [
    ((1, 8, 1, 1), _lib.KERNEL_DECODE),
    ((4, 8, 1, 1), _lib.KERNEL_DECODE),
    ((), _lib.KERNEL_DECODE),
    ((8, 1, 1), _lib.KERNEL_DECODE),
    ((1, 1, 1, 8), _lib.ERR_SCALE_SHAPE),
    ((8,), _lib.ERR_SCALE_SHAPE),
    ((2, 8, 1, 1), _lib.ERR_SCALE_SHAPE),
    ((1, 1, 1, 1, 1), _lib.ERR_RANK),
])
def test_scale_broadcasting(shape, status):
    a = _args()
    a.scale = _tensor(shape[:4] if len(shape) <= 4 else shape[:4], _lib.F32)
    if len(shape) > 4:
        a.scale.ndim = 5
    assert _select(a) == status


@pytest.mark.parametrize('shape,status', [
    ((4, 1, 1, 64), _lib.KERNEL_DECODE),
    ((4, 8, 1, 64), _lib.KERNEL_DECODE),
    ((1, 1, 1, 64), _lib.KERNEL_DECODE),
    ((64,), _lib.KERNEL_DECODE),
    ((4, 1, 1, 1), _lib.KERNEL_DECODE),
    ((4, 1, 2, 64), _lib.ERR_BIAS_QUERY),
    ((3, 64), _lib.ERR_BIAS_QUERY),
    ((4, 3, 1, 64), _lib.ERR_BIAS_SHAPE),
    ((4, 1, 1, 63), _lib.ERR_BIAS_SHAPE),
    ((2, 1, 1, 64), _lib.ERR_BIAS_SHAPE),
])
def test_key_bias_broadcasting(shape, status):
    assert _select(_args(bias_shape=shape)) == status


def test_dtype_rules():
    a = _args()
    a.k.dtype = _lib.F16
    assert _select(a) == _lib.ERR_DTYPE
    a = _args(dtype=_lib.F64)
    assert _select(a) == _lib.ERR_DTYPE
    a = _args(bias_shape=(4, 1, 1, 64), bias_dtype=_lib.F64)
    assert _select(a) == _lib.KERNEL_DECODE
    a = _args(bias_shape=(4, 1, 1, 64), bias_dtype=7)
    assert _select(a) == _lib.ERR_DTYPE


def test_shape_and_rank_rules():
    a = _args()
    a.k.size[3] = 32
    assert _select(a) == _lib.ERR_SHAPE
    a = _args()
    a.v.size[2] = 63
    assert _select(a) == _lib.ERR_SHAPE
    a = _args()
    a.q.ndim = 3
    assert _select(a) == _lib.ERR_RANK
    a = _args(d=1024, dv=64)
    assert _select(a) == _lib.ERR_UNSUPPORTED


def test_null_pointers_are_rejected():
    a = _args()
    a.scale.data = None
    assert _select(a) == _lib.ERR_NULL
    a = _args()
    a.out = None
    assert _select(a) == _lib.ERR_NULL
    assert _lib.LIB.vectra_rbf_select_kernel(None) == _lib.ERR_NULL
