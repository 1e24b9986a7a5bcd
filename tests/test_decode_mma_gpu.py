"""The tensor-core decode kernel (Nq == 1, mma.sync) against the oracle.

Serving shapes (benchmark configs 2-3) at small batch sizes, with the edge
cases of kernels/tests/test_edges.py that apply to one query per plane:
key counts that are not multiples of the 16-key boxes or the chunk, padding
masks that skip whole boxes, every key masked (NaN), far-apart points,
degenerate scales, head-transposed strided keys and values, D in {64, 128},
bf16 and fp16. Every case also runs the SIMT decode kernel as a cross-check.
"""

import numpy as np
import pytest
import torch

import vectra_b200
from tests import helpers

pytestmark = pytest.mark.gpu


def _inputs(B, H, nk, D, dtype, seed, spread=1.0):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, 1, D, generator=gen) * spread / D**0.5
    k = torch.randn(B, H, nk, D, generator=gen) * spread / D**0.5
    v = torch.randn(B, H, nk, D, generator=gen) / D**0.5
    scale = 0.1 + 0.9 * torch.rand(1, H, 1, 1, generator=gen)
    td = helpers.TORCH_DTYPES[dtype]
    return q.to(td), k.to(td), v.to(td), scale


def _run(q, k, v, scale, bias, kernel):
    args = [q.cuda(), k.cuda(), v.cuda(), scale.cuda(),
            None if bias is None else bias.cuda()]
    assert vectra_b200.kernel_for(*args, kernel=kernel) == kernel
    out = vectra_b200.rbf_attention_with_kernel(*args, kernel=kernel)
    torch.cuda.synchronize()
    return out


def _check(q, k, v, scale, bias, dtype):
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    bn = None if bias is None else bias.float().numpy()
    out = _run(q, k, v, scale, bias, 'decode_mma')
    got = out.double().cpu().numpy()
    helpers.check_eager_gate_tol(got, qn, kn, vn, scale.numpy(), bn, dtype)
    helpers.check_reference_tol(got, qn, kn, vn, scale.numpy(), bn, dtype)
    return out


@pytest.mark.parametrize('D', [64, 128])
@pytest.mark.parametrize('nk', [1, 15, 16, 17, 64, 65, 128, 200])
@pytest.mark.parametrize('dtype', ['bf16', 'f16'])
def test_matches_oracle(D, nk, dtype):
    q, k, v, scale = _inputs(6, 3, nk, D, dtype, seed=nk + D)
    _check(q, k, v, scale, None, dtype)


@pytest.mark.parametrize('D', [64, 128])
def test_padding_masks_skip_boxes(D):
    B, H, nk = 8, 4, 128
    q, k, v, scale = _inputs(B, H, nk, D, 'bf16', 3)
    bias = torch.zeros(B, 1, 1, nk)
    lengths = [1, 8, 16, 17, 40, 64, 100, 128]
    for i, L in enumerate(lengths):
        bias[i, ..., L:] = float('-inf')
    bias[3, ..., ::5] = float('-inf')          # scattered inside the prefix
    _check(q, k, v, scale, bias.bfloat16(), 'bf16')


def test_fully_masked_rows_are_nan_and_masked_rows_unused():
    B, H, nk, D = 4, 2, 96, 64
    q, k, v, scale = _inputs(B, H, nk, D, 'bf16', 4)
    bias = torch.zeros(B, 1, 1, nk)
    bias[0] = float('-inf')
    bias[2, ..., 50:] = float('-inf')
    out = _run(q, k, v, scale, bias, 'decode_mma')
    assert torch.isnan(out[0].float()).all()
    assert torch.isfinite(out[1:].float()).all()
    k2, v2 = k.clone(), v.clone()
    k2[2, :, 50:] = 300.0
    v2[2, :, 50:] = -300.0
    again = _run(q, k2, v2, scale, bias, 'decode_mma')
    # Bit-identical, NaN rows included (NaN != NaN, so compare the rows that
    # are numbers and the NaN pattern separately).
    assert torch.equal(torch.isnan(out), torch.isnan(again))
    assert torch.equal(out[1:], again[1:])


@pytest.mark.parametrize('spread', [4.0, 20.0])
def test_far_points(spread):
    q, k, v, scale = _inputs(4, 2, 200, 64, 'bf16', 5, spread)
    _check(q, k, v, scale * 0.2, None, 'bf16')


@pytest.mark.parametrize('s', [0.0, -0.01, 3.0])
def test_degenerate_and_negative_scales(s):
    q, k, v, _ = _inputs(4, 2, 70, 64, 'bf16', 6)
    _check(q, k, v, torch.tensor(s), None, 'bf16')


def test_head_transposed_keys_and_values():
    B, N, H, D = 3, 65, 4, 64
    gen = torch.Generator().manual_seed(7)
    proj = (torch.randn(B, N, 2 * H * D, generator=gen) / 8).bfloat16()
    k, v = (t.view(B, N, H, D).transpose(1, 2)
            for t in proj.cuda().split(H * D, dim=-1))
    q = (torch.randn(B, H, 1, D, generator=gen) / 8).bfloat16().cuda()
    scale = torch.full((1, H, 1, 1), 0.5)
    assert not k.is_contiguous()
    out = _run(q, k, v, scale, None, 'decode_mma')
    helpers.check_reference_tol(
        out.double().cpu().numpy(), q.float().cpu().numpy(),
        k.float().cpu().numpy(), v.float().cpu().numpy(), scale.numpy(),
        None, 'bf16')


def test_agrees_with_the_simt_decode_kernel():
    q, k, v, scale = _inputs(32, 8, 64, 64, 'bf16', 8)
    a = _run(q, k, v, scale, None, 'decode_mma').float()
    b = _run(q, k, v, scale, None, 'decode').float()
    np.testing.assert_allclose(a.cpu().numpy(), b.cpu().numpy(), rtol=2e-2,
                               atol=8e-3 * float(v.float().abs().max()))


def test_deterministic_and_shard_consistent():
    q, k, v, scale = _inputs(64, 8, 64, 64, 'bf16', 9)
    args = [t.cuda() for t in (q, k, v, scale)]
    full = vectra_b200.rbf_attention(*args)
    assert torch.equal(full, vectra_b200.rbf_attention(*args))
    for lo, hi in ((0, 16), (16, 48), (48, 64)):
        part = vectra_b200.rbf_attention(args[0][lo:hi], args[1][lo:hi],
                                         args[2][lo:hi], args[3])
        assert torch.equal(full[lo:hi], part)


def test_no_device_errors():
    from vectra_b200 import _lib  # pylint: disable=import-outside-toplevel
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.check_device_errors(stream) == _lib.OK
