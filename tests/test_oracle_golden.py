"""The oracle against the reference's own outputs (CPU only).

tests/golden/*.npz hold seeded inputs and the outputs of the reference's
four formulations (kernels/vectra_kernels/reference.py:46-161). Each oracle
function must reproduce its counterpart; the oracle is then trusted as the
checker of the CUDA path in the GPU tests.
"""

import numpy as np
import pytest

from oracle import rbf_oracle
from tests import golden

CASES = golden.names()


def _close(actual, expected, rtol, atol):
    np.testing.assert_allclose(actual, expected, rtol=rtol, atol=atol,
                               equal_nan=True)


@pytest.mark.parametrize('name', CASES)
def test_expanded_float64_matches_reference(name):
    c = golden.load(name)
    out = rbf_oracle.expanded_rbf_attention(c['q'], c['k'], c['v'],
                                            c['scale'], c['bias'])
    _close(out, c['expanded'], rtol=1e-9, atol=1e-11)


@pytest.mark.parametrize('name', CASES)
def test_eager_float32_matches_reference(name):
    c = golden.load(name)
    out = rbf_oracle.eager_rbf_attention(c['q'], c['k'], c['v'],
                                         c['scale'], c['bias'])
    _close(out, c['eager'], rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize('name', CASES)
def test_matmul_matches_reference(name):
    c = golden.load(name)
    out = rbf_oracle.round_to(
        rbf_oracle.matmul_rbf_attention(c['q'], c['k'], c['v'], c['scale'],
                                        c['bias']), c['dtype'])
    # One rounding step of the output dtype apart at most.
    tol = {'f32': 1e-4, 'f16': 2e-3, 'bf16': 1.6e-2}[c['dtype']]
    atol = tol * max(1.0, float(np.abs(c['v']).max()))
    _close(out, c['matmul'], rtol=tol, atol=atol if c['dtype'] != 'f32'
           else 2e-4)


@pytest.mark.parametrize('name', CASES)
def test_tiled_matches_reference(name):
    c = golden.load(name)
    out = rbf_oracle.round_to(
        rbf_oracle.tiled_rbf_attention(c['q'], c['k'], c['v'], c['scale'],
                                       c['bias']), c['dtype'])
    tol = {'f32': 1e-4, 'f16': 2e-3, 'bf16': 1.6e-2}[c['dtype']]
    atol = tol * max(1.0, float(np.abs(c['v']).max()))
    _close(out, c['tiled'], rtol=tol, atol=atol if c['dtype'] != 'f32'
           else 2e-4)


def test_fully_masked_rows_are_nan():
    c = golden.load('fully_masked')
    assert np.isnan(c['expanded']).all()
    out = rbf_oracle.expanded_rbf_attention(c['q'], c['k'], c['v'],
                                            c['scale'], c['bias'])
    assert np.isnan(out).all()


def test_bias_must_be_constant_across_queries():
    q = np.zeros((1, 1, 3, 4), np.float32)
    with pytest.raises(ValueError, match='constant across queries'):
        rbf_oracle.expanded_rbf_attention(q, q, q, 0.1,
                                          np.zeros((1, 1, 3, 3)))


def test_bf16_rounding_is_round_to_nearest_even():
    # 1 + 2^-8 is halfway between two bf16 values: ties go to even (1.0);
    # 1 + 3*2^-8 ties upward to 1 + 2^-6.
    x = np.array([1.0 + 2.0**-8, 1.0 + 3 * 2.0**-8, -2.5, np.inf],
                 np.float32)
    r = rbf_oracle.round_to_bf16(x)
    np.testing.assert_array_equal(r, [1.0, 1.0 + 2.0**-6, -2.5, np.inf])
    bits = rbf_oracle.bf16_bits(r)
    np.testing.assert_array_equal(rbf_oracle.from_bf16_bits(bits), r)
