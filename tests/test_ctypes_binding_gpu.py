"""The C ABI as a non-torch host binds it: the ctypes binding of the
integration guide, copied verbatim below, called with a raw CUDA stream
handle on benchmark configs 1-3's shapes and checked against the oracle;
then vectra_rbf_check_device_errors reports a clean device.

Nothing here goes through the torch binding (_vectra_rbf_torch.so): torch
only allocates the buffers and provides the stream handle, as any host's
allocator would.
"""

import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import rbf_oracle
from tests import helpers
from vectra_b200 import workloads

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# --- The integration guide's binding, verbatim (section "The C ABI"). ---
# (Its library path is relative to the repository root; the fixture below
# runs it from there.)
BINDING = r'''
import ctypes, torch
lib = ctypes.CDLL('vectra_b200/libvectra_rbf.so')

class Tensor(ctypes.Structure):
    _fields_ = [('data', ctypes.c_void_p), ('dtype', ctypes.c_int32),
                ('ndim', ctypes.c_int32), ('size', ctypes.c_int64 * 4),
                ('stride', ctypes.c_int64 * 4)]

class Args(ctypes.Structure):
    _fields_ = [('q', Tensor), ('k', Tensor), ('v', Tensor),
                ('scale', Tensor), ('key_bias', Tensor),
                ('out', ctypes.c_void_p), ('out_stride', ctypes.c_int64 * 4),
                ('flags', ctypes.c_uint32)]

DTYPE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2,
         torch.float64: 3}

def describe(t):
    d = Tensor()
    if t is not None:
        d.data, d.dtype, d.ndim = t.data_ptr(), DTYPE[t.dtype], t.dim()
        for i in range(t.dim()):
            d.size[i], d.stride[i] = t.shape[i], t.stride(i)
    return d

def rbf_attention_forward(q, k, v, scale, key_bias=None):
    out = torch.empty(*q.shape[:3], v.shape[3], dtype=v.dtype,
                      device=q.device)
    a = Args(describe(q), describe(k), describe(v), describe(scale),
             describe(key_bias), out.data_ptr())
    for i in range(4):
        a.out_stride[i] = out.stride(i)
    status = lib.vectra_rbf_attention_forward(
        ctypes.byref(a),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if status != 0:
        lib.vectra_rbf_strerror.restype = ctypes.c_char_p
        raise ValueError(lib.vectra_rbf_strerror(status).decode())
    return out
'''


@pytest.fixture(scope='module')
def binding():
    cwd = os.getcwd()
    os.chdir(ROOT)
    try:
        namespace = {}
        exec(compile(BINDING, 'integration_binding', 'exec'), namespace)  # pylint: disable=exec-used
    finally:
        os.chdir(cwd)
    return namespace


def _check(out, w, dtype):
    got = out.double().cpu().numpy()
    arrays = [None if t is None else t.float().cpu().numpy()
              for t in w.tensors()]
    want = rbf_oracle.eager_rbf_attention(*arrays)
    rtol, atol = helpers.EAGER_GATE_TOL[dtype]
    scale_v = float(np.abs(arrays[2]).max()) if dtype != 'f32' else 1.0
    helpers.assert_close(got, want, rtol, atol * scale_v)


@pytest.mark.parametrize('config,batch', [(1, None), (2, 48), (3, 40)])
def test_binding_matches_the_oracle(binding, config, batch):
    w = workloads.make(config, device='cuda', seed=9, batch=batch)
    out = binding['rbf_attention_forward'](*w.tensors())
    torch.cuda.synchronize()
    _check(out, w, w.dtype)
    lib = binding['lib']
    lib.vectra_rbf_check_device_errors.argtypes = [ctypes.c_void_p]
    assert lib.vectra_rbf_check_device_errors(
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0


def test_binding_on_a_side_stream_and_a_bad_call(binding):
    # The raw handle of a non-default stream orders the launch; a bad shape
    # comes back as the library's message, with nothing launched.
    w = workloads.make(2, device='cuda', seed=10, batch=16)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        out = binding['rbf_attention_forward'](*w.tensors())
    side.synchronize()
    _check(out, w, w.dtype)
    q, k, v, scale, _ = w.tensors()
    with pytest.raises(ValueError):
        binding['rbf_attention_forward'](q, k[:, :, :, :32], v, scale)
