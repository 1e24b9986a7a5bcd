"""The one-tile-per-plane kernels against the oracle: rbf_small (mma.sync;
Nk <= 128, Nq >= 2, D == Dv in {32, 64}, bf16/f16) and rbf_small_tc
(tcgen05 + TMEM; the same with Nq <= 96 and Nk <= 128 - D). Every test runs
on both; a case outside rbf_small_tc's range is skipped for it.

Key counts on both sides of every tile size it instantiates (32, 64, 80,
128) and query counts across one and several query blocks; the compiled
model's layout (q/k/v strided views of one [B, N, 3, H, D] projection,
benchmark config 5) with padding masks, fully masked rows (NaN) and per-head
biases; degenerate scales; agreement with the generic kernel; determinism
and batch-slice consistency. Tolerances are the reference suite's
(kernels/tests/test_parity.py:33-37) and north_star's eager gate.
"""

import numpy as np
import pytest
import torch

import vectra_b200
from tests import helpers

pytestmark = pytest.mark.gpu

SMALL_KERNELS = ['small', 'small_tc']


@pytest.fixture(params=SMALL_KERNELS)
def kernel(request):
    return request.param


def _inputs(B, H, nq, nk, D, dtype, seed, spread=1.0):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, nq, D, generator=gen) * spread / D**0.5
    k = torch.randn(B, H, nk, D, generator=gen) * spread / D**0.5
    v = torch.randn(B, H, nk, D, generator=gen) / D**0.5
    scale = 0.2 + 1.5 * torch.rand(1, H, 1, 1, generator=gen)
    td = helpers.TORCH_DTYPES[dtype]
    return q.to(td), k.to(td), v.to(td), scale


def _run(q, k, v, scale, bias, kernel='small'):
    args = [t.cuda() for t in (q, k, v, scale)]
    args.append(None if bias is None else bias.cuda())
    if kernel == 'small_tc':
        try:
            vectra_b200.kernel_for(*args, kernel=kernel)
        except ValueError:
            pytest.skip('outside rbf_small_tc (Nq <= 96, Nk <= 128 - D)')
    assert vectra_b200.kernel_for(*args, kernel=kernel) == kernel
    out = vectra_b200.rbf_attention_with_kernel(*args, kernel=kernel)
    torch.cuda.synchronize()
    return out


def _check(q, k, v, scale, bias, dtype, kernel='small'):
    out = _run(q, k, v, scale, bias, kernel)
    got = out.double().cpu().numpy()
    qn, kn, vn = (t.float().cpu().numpy() for t in (q, k, v))
    bn = None if bias is None else bias.float().cpu().numpy()
    helpers.check_reference_tol(got, qn, kn, vn, scale.numpy(), bn, dtype)
    helpers.check_eager_gate_tol(got, qn, kn, vn, scale.numpy(), bn, dtype)
    return out


@pytest.mark.parametrize('nk', [1, 15, 16, 17, 32, 33, 64, 65, 80, 81, 127,
                                128])
@pytest.mark.parametrize('D', [32, 64])
@pytest.mark.parametrize('dtype', ['bf16', 'f16'])
def test_key_counts_match_oracle(nk, D, dtype, kernel):
    q, k, v, scale = _inputs(3, 2, 20, nk, D, dtype, seed=nk + D)
    _check(q, k, v, scale, None, dtype, kernel)


@pytest.mark.parametrize('nq', [2, 15, 16, 17, 31, 32, 33, 64, 65, 95, 96,
                                128, 129, 300])
def test_query_counts_match_oracle(nq, kernel):
    q, k, v, scale = _inputs(2, 3, nq, 65, 32, 'bf16', seed=nq)
    _check(q, k, v, scale, None, 'bf16', kernel)


def _model_layout(B, N, H, D, dtype, seed):
    """q, k, v as the compiled model passes them: head-transposed views of
    one [B, N, 3, H, D] projection (row stride 3 H D)."""
    gen = torch.Generator().manual_seed(seed)
    qkv = (torch.randn(B, N, 3, H, D, generator=gen) / D**0.5)
    qkv = qkv.to(helpers.TORCH_DTYPES[dtype]).cuda()
    q, k, v = qkv.permute(2, 0, 3, 1, 4)
    return q, k, v


@pytest.mark.parametrize('dtype', ['bf16', 'f16'])
def test_compiled_model_layout_with_padding(dtype, kernel):
    B, N, H, D = 12, 65, 8, 32
    q, k, v = _model_layout(B, N, H, D, dtype, 3)
    assert not q.is_contiguous() and q.stride() == (N * 3 * H * D, D,
                                                     3 * H * D, 1)
    gen = torch.Generator().manual_seed(4)
    scale = 1.0 / (2.0 * (0.5 + torch.rand(1, H, 1, 1, generator=gen)) ** 2)
    valid = torch.randint(9, N + 1, (B,), generator=gen)
    bias = torch.zeros(B, 1, 1, N)
    for b in range(B):
        bias[b, ..., valid[b]:] = float('-inf')
    bias = bias.to(helpers.TORCH_DTYPES[dtype])
    _check(q, k, v, scale, bias, dtype, kernel)


def test_fully_masked_rows_are_nan_and_masked_keys_unused(kernel):
    B, H, nq, nk, D = 4, 2, 33, 70, 32
    q, k, v, scale = _inputs(B, H, nq, nk, D, 'bf16', 5)
    bias = torch.zeros(B, 1, 1, nk)
    bias[0] = float('-inf')
    bias[2, ..., 40:] = float('-inf')
    out = _run(q, k, v, scale, bias, kernel)
    assert torch.isnan(out[0].float()).all()
    assert torch.isfinite(out[1:].float()).all()
    k2, v2 = k.clone(), v.clone()
    k2[2, :, 40:] = 300.0
    v2[2, :, 40:] = -300.0
    again = _run(q, k2, v2, scale, bias, kernel)
    assert torch.equal(torch.isnan(out), torch.isnan(again))
    assert torch.equal(out[1:], again[1:])


def test_per_head_bias_and_per_row_scale(kernel):
    B, H, nq, nk, D = 3, 4, 17, 50, 64
    q, k, v, _ = _inputs(B, H, nq, nk, D, 'f16', 6)
    gen = torch.Generator().manual_seed(7)
    bias = torch.randn(B, H, 1, nk, generator=gen)
    bias[:, 1, :, 30:] = float('-inf')
    scale = 0.1 + torch.rand(B, H, 1, 1, generator=gen)
    _check(q, k, v, scale, bias.half(), 'f16', kernel)


@pytest.mark.parametrize('s', [0.0, -0.01, 3.0])
def test_degenerate_and_negative_scales(s, kernel):
    q, k, v, _ = _inputs(3, 2, 20, 40, 32, 'bf16', 8)
    _check(q, k, v, torch.tensor(s), None, 'bf16', kernel)


@pytest.mark.parametrize('spread', [4.0, 20.0])
def test_far_points(spread, kernel):
    q, k, v, scale = _inputs(3, 2, 20, 65, 32, 'bf16', 9, spread)
    _check(q, k, v, scale * 0.05, None, 'bf16', kernel)


def test_agrees_with_the_generic_kernel(kernel):
    q, k, v = _model_layout(16, 65, 8, 32, 'bf16', 10)
    scale = torch.full((1, 8, 1, 1), 0.7)
    a = _run(q, k, v, scale, None, kernel).float()
    b = _run(q, k, v, scale, None, kernel='generic').float()
    np.testing.assert_allclose(a.cpu().numpy(), b.cpu().numpy(), rtol=2e-2,
                               atol=8e-3 * float(v.float().abs().max()))


def test_deterministic_and_batch_slices_agree(kernel):
    q, k, v = _model_layout(40, 65, 8, 32, 'bf16', 11)
    scale = torch.full((1, 8, 1, 1), 0.4).cuda()

    def run(*a):
        return vectra_b200.rbf_attention_with_kernel(*a, kernel=kernel)
    full = run(q, k, v, scale)
    assert torch.equal(full, run(q, k, v, scale))
    for lo, hi in ((0, 7), (7, 33), (33, 40)):
        part = run(q[lo:hi], k[lo:hi], v[lo:hi], scale)
        assert torch.equal(full[lo:hi], part)


def test_model_site_selects_the_mma_sync_kernel():
    # rbf_small_tc runs only when forced (slower on this shape).
    q, k, v = _model_layout(4, 65, 8, 32, 'bf16', 12)
    scale = torch.full((1, 8, 1, 1), 0.4).cuda()
    assert vectra_b200.kernel_for(q, k, v, scale) == 'small'
    assert vectra_b200.kernel_for(q, k, v, scale, kernel='small_tc') == (
        'small_tc')
    q2, k2, v2 = _model_layout(4, 97, 8, 32, 'bf16', 12)
    with pytest.raises(ValueError):
        vectra_b200.kernel_for(q2, k2, v2, scale, kernel='small_tc')


def test_the_two_kernels_agree_on_the_model_site():
    # Same inputs, same rounding of P to bf16: the kernels differ only in
    # the order of the fp32 sums (mma.sync fragments vs tcgen05).
    q, k, v = _model_layout(64, 65, 8, 32, 'bf16', 13)
    gen = torch.Generator().manual_seed(14)
    scale = (0.1 + torch.rand(1, 8, 1, 1, generator=gen)).cuda()
    bias = torch.zeros(64, 1, 1, 65)
    bias[::3, ..., 40:] = float('-inf')
    bias = bias.bfloat16().cuda()
    a = vectra_b200.rbf_attention_with_kernel(q, k, v, scale, bias,
                                              kernel='small').float()
    b = vectra_b200.rbf_attention_with_kernel(q, k, v, scale, bias,
                                              kernel='small_tc').float()
    np.testing.assert_allclose(a.cpu().numpy(), b.cpu().numpy(), rtol=2e-2,
                               atol=4e-3 * float(v.float().abs().max()))


def test_no_device_errors():
    from vectra_b200 import _lib  # pylint: disable=import-outside-toplevel
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.check_device_errors(stream) == _lib.OK
