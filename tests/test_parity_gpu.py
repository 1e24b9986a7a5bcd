"""Parity of the CUDA operator with the reference (B200 only).

Two anchors:
* the golden vectors: outputs of the reference's own float64 oracle
  (kernels/vectra_kernels/reference.py:61-76) on seeded inputs, stored in
  tests/golden/ — the CUDA result must match them directly;
* the NumPy oracle (pinned to those vectors by test_oracle_golden.py) on the
  reference test suite's full shapes (kernels/tests/test_parity.py:39-46).

Every case runs through the automatic kernel choice and through each kernel
that accepts it, so a specialised kernel can never hide behind the generic
one.
"""

import numpy as np
import pytest
import torch

import vectra_b200
from tests import golden
from tests import helpers

pytestmark = pytest.mark.gpu

# Reference test shapes (B, H, Nq, Nk, D, Dv), kernels/tests/test_parity.py.
SHAPES = [
    (8, 8, 65, 65, 32, 32),
    (2, 4, 257, 257, 64, 64),
    (1, 1, 16, 16, 16, 16),
    (4, 2, 33, 129, 64, 32),
]
# Serving-style shapes (Nq == 1) that the decode kernel takes.
DECODE_SHAPES = [
    (8, 4, 1, 16, 32, 32),
    (16, 8, 1, 64, 64, 64),
    (5, 3, 1, 200, 64, 64),
    (4, 8, 1, 65, 128, 128),
    (6, 2, 1, 129, 32, 32),
]


def _kernels_for(q_shape, d, dv, dtype, nk):
    kernels = ['auto', 'generic']
    if q_shape[2] == 1 and d == dv and (
            d in (32, 64, 128) if dtype != 'f32' else d in (32, 64)):
        kernels.append('decode')
    if (q_shape[2] >= 2 and nk <= 128 and d == dv and d in (32, 64)
            and dtype != 'f32'):
        kernels.append('small')
        if q_shape[2] <= 96 and nk <= 128 - d:
            kernels.append('small_tc')
    return kernels


def _case_tol(name, dtype, v):
    rtol, atol = helpers.REFERENCE_TOL[dtype]
    atol *= float(np.abs(v).max())
    if name == 'far' or name.startswith('scale_'):
        atol = max(atol, 1e-4)  # kernels/tests/test_edges.py:84-100
    return rtol, atol


@pytest.mark.parametrize('name', golden.names())
def test_matches_reference_golden_vectors(name):
    c = golden.load(name)
    q, k, v = c['q'], c['k'], c['v']
    for kernel in _kernels_for(q.shape, q.shape[3], v.shape[3], c['dtype'],
                               k.shape[2]):
        out = helpers.run(q, k, v, c['scale'], c['bias'], c['dtype'],
                          kernel=kernel)
        rtol, atol = _case_tol(name, c['dtype'], v)
        helpers.assert_close(out, c['expanded'], rtol, atol)


@pytest.mark.parametrize('shape', SHAPES + DECODE_SHAPES)
@pytest.mark.parametrize('dtype', ['f32', 'f16', 'bf16'])
@pytest.mark.parametrize('with_bias', [False, True])
def test_matches_float64_oracle(shape, dtype, with_bias):
    q, k, v, scale, bias = helpers.parity_inputs(shape, dtype, 0, with_bias)
    for kernel in _kernels_for(q.shape, shape[4], shape[5], dtype, shape[3]):
        out = helpers.run(q, k, v, scale, bias, dtype, kernel=kernel)
        helpers.check_reference_tol(out, q, k, v, scale, bias, dtype)
        helpers.check_eager_gate_tol(out, q, k, v, scale, bias, dtype)


def test_output_dtype_shape_and_device():
    q, k, v, scale, bias = helpers.parity_inputs(SHAPES[0], 'bf16', 2, True)
    out = vectra_b200.rbf_attention(
        helpers.to_cuda(q, 'bf16'), helpers.to_cuda(k, 'bf16'),
        helpers.to_cuda(v, 'bf16'), helpers.to_cuda(scale),
        helpers.to_cuda(bias))
    assert out.shape == (8, 8, 65, 32)
    assert out.dtype == torch.bfloat16 and out.is_cuda


def test_custom_op_dispatches_and_matches():
    # kernels/tests/test_parity.py:90-98, on the GPU.
    q, k, v, scale, bias = helpers.parity_inputs(SHAPES[0], 'f32', 2, True)
    out = torch.ops.vectra.rbf_attention(
        helpers.to_cuda(q), helpers.to_cuda(k), helpers.to_cuda(v),
        helpers.to_cuda(scale), helpers.to_cuda(bias))
    from oracle import rbf_oracle  # pylint: disable=import-outside-toplevel
    helpers.assert_close(
        out.double().cpu().numpy(),
        rbf_oracle.expanded_rbf_attention(q, k, v, scale, bias), 1e-4, 1e-5)
