"""Failure detection on the GPU, without faulting it.

Every wait in the kernels is bounded: when one runs out the kernel records
the timeout in the device error word and returns, and the host reads it
through vectra_rbf_check_device_errors. The self-test kernel makes such a
wait run out for real (an mbarrier that nothing completes) and the context
must stay usable afterwards. Guard bands around caller-owned output buffers
catch out-of-bounds stores of every kernel.
"""

import ctypes

import pytest
import torch

import vectra_b200
from vectra_b200 import _lib

pytestmark = pytest.mark.gpu


def test_a_wait_that_runs_out_is_reported_and_the_context_survives():
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.check_device_errors(stream) == _lib.OK
    assert _lib.selftest_wait_timeout(stream) == _lib.OK
    assert _lib.check_device_errors(stream) == _lib.ERR_DEVICE
    assert _lib.check_device_errors(stream) == _lib.OK  # read and cleared
    # The context still runs kernels correctly.
    q = torch.randn(4, 2, 1, 64, device='cuda').bfloat16()
    k = torch.randn(4, 2, 16, 64, device='cuda').bfloat16()
    v = torch.randn(4, 2, 16, 64, device='cuda').bfloat16()
    out = vectra_b200.rbf_attention(q, k, v, torch.ones(1, 2, 1, 1).cuda())
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert _lib.check_device_errors(stream) == _lib.OK


def _describe(t):
    d = _lib.Tensor()
    if t is None:
        return d
    d.data = t.data_ptr()
    d.dtype = {torch.float32: _lib.F32, torch.float16: _lib.F16,
               torch.bfloat16: _lib.BF16}[t.dtype]
    d.ndim = t.dim()
    for i in range(t.dim()):
        d.size[i] = t.shape[i]
        d.stride[i] = t.stride(i)
    return d


CASES = {
    'decode': ((6, 3, 1, 70, 64), 'bf16', True),
    # Bias rows of 72 and 200 float32 keys are whole 16-byte runs: the
    # byte-ring kernel for biased problems (one and two chunks per plane).
    'decode_masked': ((6, 3, 1, 72, 64), 'bf16', True),
    'decode_masked_2chunks': ((5, 2, 1, 200, 64), 'bf16', True),
    'small': ((3, 2, 33, 65, 32), 'bf16', True),
    'small_tc': ((3, 2, 33, 65, 32), 'bf16', True),
    'tc': ((1, 2, 300, 200, 64), 'bf16', True),
    'generic': ((2, 3, 21, 37, 48), 'f32', True),
}


@pytest.mark.parametrize('kernel', sorted(CASES))
def test_output_guard_bands_are_untouched(kernel):
    (B, H, nq, nk, D), dtype, with_bias = CASES[kernel]
    td = {'bf16': torch.bfloat16, 'f16': torch.float16,
          'f32': torch.float32}[dtype]
    gen = torch.Generator(device='cuda').manual_seed(3)
    q = torch.randn(B, H, nq, D, device='cuda', generator=gen).to(td)
    k = torch.randn(B, H, nk, D, device='cuda', generator=gen).to(td)
    v = torch.randn(B, H, nk, D, device='cuda', generator=gen).to(td)
    scale = torch.full((1, H, 1, 1), 0.1, device='cuda')
    bias = torch.zeros(B, 1, 1, nk, device='cuda')
    bias[0, ..., nk // 2:] = float('-inf')
    # The output sits inside a larger buffer filled with a canary pattern;
    # rows are padded too (row stride D + 8 elements keeps 16-byte
    # alignment for every dtype here).
    guard = 4096
    row = D + 8
    n_out = B * H * nq * row
    buf = torch.full((guard + n_out + guard,), 7.0, device='cuda', dtype=td)
    out = buf[guard:guard + n_out].view(B, H, nq, row)[..., :D]
    a = _lib.Args()
    a.q, a.k, a.v = _describe(q), _describe(k), _describe(v)
    a.scale = _describe(scale)
    a.key_bias = _describe(bias if with_bias else None)
    a.out = out.data_ptr()
    for i in range(4):
        a.out_stride[i] = out.stride(i)
    a.flags = {'decode': _lib.FLAG_FORCE_DECODE,
               'decode_masked': _lib.FLAG_FORCE_DECODE,
               'decode_masked_2chunks': _lib.FLAG_FORCE_DECODE,
               'small': _lib.FLAG_FORCE_SMALL,
               'small_tc': _lib.FLAG_FORCE_SMALL_TC,
               'tc': _lib.FLAG_FORCE_TC,
               'generic': _lib.FLAG_FORCE_GENERIC}[kernel]
    assert _lib.LIB.vectra_rbf_select_kernel(ctypes.byref(a)) >= 0, kernel
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.LIB.vectra_rbf_attention_forward(
        ctypes.byref(a), ctypes.c_void_p(stream)) == _lib.OK
    torch.cuda.synchronize()
    assert _lib.check_device_errors(stream) == _lib.OK
    assert bool((buf[:guard] == 7).all()) and bool((buf[-guard:] == 7).all())
    pad = buf[guard:guard + n_out].view(B, H, nq, row)[..., D:]
    assert bool((pad == 7).all()), 'a kernel wrote into the row padding'
    ref = vectra_b200.rbf_attention_with_kernel(
        q, k, v, scale, bias if with_bias else None, kernel='generic')
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2,
                               atol=2e-2, equal_nan=True)
