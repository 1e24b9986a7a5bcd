"""The byte-ring decode kernel for biased problems against the oracle.

Nq == 1 with a key bias whose rows are whole 16-byte runs (f32, f16 or
bf16 elements, unit key stride) goes to rbf_decode_masked_kernel: each
(query, head) plane's chunk is copied at its live size (key rows between
its first and last finite bias). The cases cover the variable key counts
of benchmark config 3, holes inside the live range, fully masked and
single-key planes, per-head biases, every bias dtype, one and several
chunks per plane, f32/f16/bf16 inputs, many planes per block (the ring
wraps many times) and the reference suite's tolerances
(kernels/tests/test_parity.py:33-37) plus north_star's eager gate.
"""

import pytest
import torch

import vectra_b200
from tests import helpers

pytestmark = pytest.mark.gpu


def _case(B, H, nk, D, dtype, bias_dtype, seed, heads_in_bias=1,
          holes=False, lengths=None):
    gen = torch.Generator().manual_seed(seed)
    td = helpers.TORCH_DTYPES[dtype]
    q = (torch.randn(B, H, 1, D, generator=gen) / D**0.5).to(td)
    k = (torch.randn(B, H, nk, D, generator=gen) / D**0.5).to(td)
    v = (torch.randn(B, H, nk, D, generator=gen) / D**0.5).to(td)
    scale = 0.1 + torch.rand(1, H, 1, 1, generator=gen)
    if lengths is None:
        lengths = torch.randint(1, nk + 1, (B,), generator=gen)
    bias = torch.zeros(B, heads_in_bias, 1, nk)
    for b in range(B):
        bias[b, ..., int(lengths[b]):] = float('-inf')
    if holes:  # masked keys inside the live range
        bias[:, ..., 1::3] = float('-inf')
    return q, k, v, scale, bias.to(helpers.TORCH_DTYPES[bias_dtype])


def _check(q, k, v, scale, bias, dtype):
    args = [t.cuda() for t in (q, k, v, scale, bias)]
    assert vectra_b200.kernel_for(*args) == 'decode'
    out = vectra_b200.rbf_attention(*args)
    torch.cuda.synchronize()
    got = out.double().cpu().numpy()
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    bn = bias.float().numpy()
    helpers.check_reference_tol(got, qn, kn, vn, scale.numpy(), bn, dtype)
    helpers.check_eager_gate_tol(got, qn, kn, vn, scale.numpy(), bn, dtype)
    return out


@pytest.mark.parametrize('nk', [8, 16, 64, 72, 128, 136, 256, 1000])
@pytest.mark.parametrize('dtype', ['bf16', 'f16'])
def test_variable_counts_match_oracle(nk, dtype):
    _check(*_case(40, 4, nk, 64, dtype, 'f32', seed=nk), dtype)


@pytest.mark.parametrize('bias_dtype', ['f32', 'f16', 'bf16'])
def test_every_bias_dtype(bias_dtype):
    _check(*_case(33, 8, 128, 64, 'bf16', bias_dtype, seed=7), 'bf16')


def test_holes_inside_the_live_range():
    _check(*_case(25, 8, 128, 64, 'bf16', 'bf16', seed=8, holes=True),
           'bf16')


def test_per_head_bias():
    _check(*_case(17, 4, 96, 64, 'f16', 'f32', seed=9, heads_in_bias=4),
           'f16')


@pytest.mark.parametrize('D', [32, 64, 128])
def test_head_widths(D):
    _check(*_case(20, 3, 128, D, 'bf16', 'bf16', seed=D), 'bf16')


def test_f32_inputs():
    _check(*_case(20, 4, 64, 64, 'f32', 'f32', seed=11), 'f32')


def test_fully_masked_and_single_key_planes():
    lengths = torch.tensor([0, 1, 128, 0, 2, 64, 1])
    q, k, v, scale, bias = _case(7, 2, 128, 64, 'bf16', 'bf16', seed=12,
                                 lengths=lengths)
    out = vectra_b200.rbf_attention(*[t.cuda() for t in
                                      (q, k, v, scale, bias)]).float().cpu()
    assert torch.isnan(out[0]).all() and torch.isnan(out[3]).all()
    # One live key: the output is that key's value row.
    torch.testing.assert_close(out[1, :, 0], v[1, :, 0].float(), rtol=0,
                               atol=0)
    live = [1, 2, 4, 5, 6]
    _check(q[live], k[live], v[live], scale, bias[live], 'bf16')


def test_many_planes_per_block_wrap_the_ring():
    # 16,384 planes over 148 blocks: ~110 items per block through ring
    # quarters that hold a handful of items each.
    _check(*_case(2048, 8, 128, 64, 'bf16', 'bf16', seed=13), 'bf16')


def test_agrees_with_the_fixed_stage_path():
    # A bias of 127 float32 keys is not a whole 16-byte run, so it takes
    # the fixed-stage kernel; the same problem with one masked key appended
    # (128 keys) takes the byte ring. The masked key changes nothing.
    q, k, v, scale, bias = _case(30, 4, 128, 64, 'bf16', 'f32', seed=14)
    bias[..., 127] = float('-inf')
    full = vectra_b200.rbf_attention(*[t.cuda() for t in
                                       (q, k, v, scale, bias)])
    cut = vectra_b200.rbf_attention(
        *[t.cuda() for t in (q, k[:, :, :127].contiguous(),
                             v[:, :, :127].contiguous(), scale,
                             bias[..., :127].contiguous())])
    torch.testing.assert_close(full, cut, rtol=2e-2, atol=2e-2,
                               equal_nan=True)


def test_deterministic():
    args = [t.cuda() for t in _case(300, 8, 128, 64, 'bf16', 'bf16',
                                    seed=15)]
    a = vectra_b200.rbf_attention(*args)
    b = vectra_b200.rbf_attention(*args)
    assert torch.equal(torch.isnan(a), torch.isnan(b))
    assert torch.equal(a.nan_to_num(), b.nan_to_num())
