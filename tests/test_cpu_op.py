"""The operator's CPU implementation (vectra_b200/csrc/rbf_cpu.cpp) against
the reference's own outputs and the oracle.

CPU tensors dispatch to it, as the reference's default implementation runs
them (kernels/vectra_kernels/custom_ops.py:52-72 ->
reference.matmul_rbf_attention, reference.py:79-99): float32 arithmetic,
the result in v's dtype, key_bias broadcast like `logits + key_bias`.
Golden vectors (tests/golden) hold the reference's matmul result; the
tolerance is the golden matmul test's (one rounding step of the output
dtype, against a reference that formed distances by expansion).
"""

import numpy as np
import pytest
import torch

import vectra_b200
from oracle import rbf_oracle
from tests import golden

TORCH = {'f32': torch.float32, 'f16': torch.float16, 'bf16': torch.bfloat16}
TOL = {'f32': 1e-4, 'f16': 2e-3, 'bf16': 1.6e-2}


def _cpu(a, dtype):
    return None if a is None else torch.from_numpy(
        np.asarray(a, np.float32)).to(TORCH[dtype])


@pytest.mark.parametrize('name', golden.names())
def test_cpu_op_matches_reference_matmul(name):
    c = golden.load(name)
    dt = c['dtype']
    scale = torch.as_tensor(np.asarray(c['scale'], np.float32))
    bias = None if c['bias'] is None else _cpu(c['bias'], 'f32')
    out = torch.ops.vectra.rbf_attention(
        _cpu(c['q'], dt), _cpu(c['k'], dt), _cpu(c['v'], dt), scale, bias)
    assert out.dtype == TORCH[dt] and out.device.type == 'cpu'
    assert out.shape == c['matmul'].shape
    tol = TOL[dt]
    atol = (2e-4 if dt == 'f32'
            else tol * max(1.0, float(np.abs(c['v']).max())))
    np.testing.assert_allclose(out.float().numpy(), c['matmul'], rtol=tol,
                               atol=atol, equal_nan=True)


def test_cpu_op_matches_float64_oracle_on_strided_inputs():
    # q, k, v as head-split views of one [B, N, 3, H, D] projection (the
    # compiled model's layout), bias [B, 1, 1, N]: the output follows q's
    # layout as on CUDA, values match the float64 oracle.
    gen = torch.Generator().manual_seed(4)
    b, n, h, d = 3, 21, 4, 16
    qkv = torch.randn(b, n, 3, h, d, generator=gen)
    q, k, v = qkv.permute(2, 0, 3, 1, 4)
    scale = 0.05 + 0.3 * torch.rand(1, h, 1, 1, generator=gen)
    bias = torch.zeros(b, 1, 1, n)
    bias[1, ..., 15:] = float('-inf')
    out = torch.ops.vectra.rbf_attention(q, k, v, scale, bias)
    assert out.stride() == vectra_b200.custom_ops.output_strides(q, d)
    want = rbf_oracle.expanded_rbf_attention(
        q.numpy(), k.numpy(), v.numpy(), scale.numpy(), bias.numpy())
    np.testing.assert_allclose(out.double().numpy(), want, rtol=1e-4,
                               atol=1e-5)


def test_cpu_op_edge_cases():
    gen = torch.Generator().manual_seed(5)
    q = torch.randn(2, 3, 4, 8, generator=gen)
    k = torch.randn(2, 3, 6, 8, generator=gen)
    v = torch.randn(2, 3, 6, 5, generator=gen)
    scale = torch.tensor(0.2)  # 0-dim, broadcast to every plane
    # Every key masked for batch row 1: NaN rows, as softmax gives.
    bias = torch.zeros(2, 1, 1, 6)
    bias[1] = float('-inf')
    out = torch.ops.vectra.rbf_attention(q, k, v, scale, bias)
    assert torch.isnan(out[1]).all() and not torch.isnan(out[0]).any()
    # A bias that varies across queries broadcasts on CPU, as the
    # reference's CPU formulation allows (the CUDA path rejects it).
    qbias = torch.randn(2, 1, 4, 6, generator=gen)
    got = torch.ops.vectra.rbf_attention(q, k, v, scale, qbias)
    for i in range(4):  # one query at a time: its bias row is constant
        want = rbf_oracle.eager_rbf_attention(
            q[:, :, i:i + 1].numpy(), k.numpy(), v.numpy(), scale.numpy(),
            qbias[:, :, i:i + 1].numpy())
        np.testing.assert_allclose(got[:, :, i:i + 1].numpy(), want,
                                   rtol=1e-5, atol=1e-6)
    # No keys: an empty weighted sum is zero.
    empty = torch.ops.vectra.rbf_attention(q, k[:, :, :0], v[:, :, :0],
                                           scale)
    assert empty.shape == (2, 3, 4, 5) and (empty == 0).all()
    # Zero and negative coefficients are legal.
    for g in (0.0, -0.01):
        got = torch.ops.vectra.rbf_attention(q, k, v, torch.tensor(g))
        want = rbf_oracle.expanded_rbf_attention(q.numpy(), k.numpy(),
                                                 v.numpy(), g)
        np.testing.assert_allclose(got.double().numpy(), want, rtol=1e-5,
                                   atol=1e-6)
    with pytest.raises(ValueError, match='broadcastable'):
        torch.ops.vectra.rbf_attention(q, k, v, torch.rand(2, 3, 4, 1))
    with pytest.raises(ValueError, match='rank 4'):
        torch.ops.vectra.rbf_attention(q[0], k[0], v[0], scale)


def test_cpu_op_opcheck():
    gen = torch.Generator().manual_seed(6)
    q = torch.randn(2, 3, 5, 16, generator=gen)
    k = torch.randn(2, 3, 9, 16, generator=gen)
    v = torch.randn(2, 3, 9, 8, generator=gen)
    scale = torch.rand(1, 3, 1, 1, generator=gen) * 0.1 + 0.02
    bias = torch.zeros(2, 1, 1, 9)
    bias[1, ..., 7:] = float('-inf')
    torch.library.opcheck(
        torch.ops.vectra.rbf_attention.default, (q, k, v, scale, bias),
        test_utils=('test_schema', 'test_faketensor',
                    'test_aot_dispatch_static', 'test_aot_dispatch_dynamic'))
    # And with the head-transposed layout the fake implementation declares.
    qkv = torch.randn(2, 7, 3, 3, 16, generator=gen)
    qs, ks, vs = qkv.permute(2, 0, 3, 1, 4)
    torch.library.opcheck(
        torch.ops.vectra.rbf_attention.default, (qs, ks, vs, scale, None),
        test_utils=('test_schema', 'test_faketensor'))
