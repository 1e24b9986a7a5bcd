"""Helpers for the GPU parity tests: seeded inputs, running the operator,
and the tolerance rules.

Tolerances (all written here, used by every parity test):

* Reference test matrix against the float64 oracle
  (kernels/tests/test_parity.py:33-37): rtol / atol x max|V| of
  fp32 (1e-4, 1e-5), fp16 (1e-3, 1e-3), bf16 (1e-2, 8e-3).
* Acceptance gate against the eager fp32 formulation: fp32 I/O rtol 1e-3,
  atol 1e-5; bf16 (and fp16) I/O rtol 2e-2 with the reference's half
  precision atol 8e-3 x max|V| (a relative bound alone is meaningless for
  outputs near zero).
"""

import numpy as np
import torch

from oracle import rbf_oracle

TORCH_DTYPES = {'f32': torch.float32, 'f16': torch.float16,
                'bf16': torch.bfloat16}

REFERENCE_TOL = {'f32': (1e-4, 1e-5), 'f16': (1e-3, 1e-3),
                 'bf16': (1e-2, 8e-3)}
EAGER_GATE_TOL = {'f32': (1e-3, 1e-5), 'f16': (2e-2, 8e-3),
                'bf16': (2e-2, 8e-3)}


def to_cuda(a, dtype='f32'):
    if a is None:
        return None
    return torch.as_tensor(np.asarray(a, np.float32)).to(
        'cuda', TORCH_DTYPES[dtype])


def run(q, k, v, scale, bias=None, dtype='f32', kernel='auto',
        bias_dtype=None):
    """Runs the operator on CUDA from NumPy inputs; returns float64 NumPy."""
    import vectra_b200  # pylint: disable=import-outside-toplevel
    args = (to_cuda(q, dtype), to_cuda(k, dtype), to_cuda(v, dtype),
            to_cuda(scale, 'f32'),
            to_cuda(bias, bias_dtype or 'f32') if bias is not None else None)
    if kernel == 'auto':
        out = vectra_b200.rbf_attention(*args)
    else:
        out = vectra_b200.rbf_attention_with_kernel(*args, kernel=kernel)
    torch.cuda.synchronize()
    return out.double().cpu().numpy()


def assert_close(actual, expected, rtol, atol):
    np.testing.assert_allclose(actual, expected, rtol=rtol, atol=atol,
                               equal_nan=True)


def check_reference_tol(actual, q, k, v, scale, bias, dtype):
    """The reference's own gate: float64 oracle, tolerance x max|V|."""
    expected = rbf_oracle.expanded_rbf_attention(q, k, v, scale, bias)
    rtol, atol = REFERENCE_TOL[dtype]
    assert_close(actual, expected, rtol, atol * float(np.abs(v).max()))


def check_eager_gate_tol(actual, q, k, v, scale, bias, dtype):
    """The acceptance gate: the eager fp32 formulation."""
    expected = rbf_oracle.eager_rbf_attention(q, k, v, scale, bias)
    rtol, atol = EAGER_GATE_TOL[dtype]
    if dtype != 'f32':
        atol *= float(np.abs(v).max())
    assert_close(actual, expected, rtol, atol)


def parity_inputs(shape, dtype, seed, with_bias):
    """kernels/tests/test_parity.py:48-63 `_inputs`, as NumPy arrays with
    values rounded to `dtype`."""
    batch, heads, n_q, n_k, dim, value_dim = shape
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, heads, n_q, dim, generator=gen)
    k = torch.randn(batch, heads, n_k, dim, generator=gen)
    v = torch.randn(batch, heads, n_k, value_dim, generator=gen)
    scale = 1.0 / (2.0 * dim * (0.5 + torch.rand(1, heads, 1, 1,
                                                  generator=gen)))
    bias = None
    if with_bias:
        bias = torch.zeros(batch, 1, 1, n_k)
        bias[:, :, :, n_k // 2 + 1:] = float('-inf')
    rnd = lambda t: rbf_oracle.round_to(t.numpy(), dtype)  # noqa: E731
    return (rnd(q), rnd(k), rnd(v), scale.numpy(),
            None if bias is None else bias.numpy())
