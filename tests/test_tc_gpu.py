"""The tensor-core kernel (tcgen05 + TMEM) against the oracle (B200 only).

Long-sequence self-attention shapes (benchmark config 4 is B=16, H=16,
L=4096, D=128, bf16) at sizes the oracle finishes quickly, with the edge
cases of kernels/tests/test_edges.py that apply to this path: tails that are
not multiples of the 128-row tiles, padding masks, fully masked rows,
far-apart points (exercising the lazy O rescaling), degenerate scales and
head-transposed strided views.
"""

import numpy as np
import pytest
import torch

import vectra_b200
from oracle import rbf_oracle
from tests import helpers

pytestmark = pytest.mark.gpu


def _inputs(B, H, nq, nk, D, dtype, seed, spread=1.0):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, nq, D, generator=gen) * spread / D**0.5
    k = torch.randn(B, H, nk, D, generator=gen) * spread / D**0.5
    v = torch.randn(B, H, nk, D, generator=gen) / D**0.5
    scale = 0.01 + 0.19 * torch.rand(1, H, 1, 1, generator=gen)
    td = helpers.TORCH_DTYPES[dtype]
    return q.to(td), k.to(td), v.to(td), scale


def _check(out, q, k, v, scale, bias, dtype, rows=None):
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    bn = None if bias is None else bias.float().numpy()
    got = out.double().cpu().numpy()
    if rows is not None:
        qn, got = qn[:, :, rows], got[:, :, rows]
    helpers.check_eager_gate_tol(got, qn, kn, vn, scale.numpy(), bn, dtype)
    helpers.check_reference_tol(got, qn, kn, vn, scale.numpy(), bn, dtype)


def _run(q, k, v, scale, bias=None, kernel='tc'):
    args = [q.cuda(), k.cuda(), v.cuda(), scale.cuda(),
            None if bias is None else bias.cuda()]
    assert vectra_b200.kernel_for(*args, kernel=kernel) == 'tc'
    out = vectra_b200.rbf_attention_with_kernel(*args, kernel=kernel)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize('shape', [
    (1, 1, 128, 128, 128), (1, 1, 128, 128, 64), (2, 3, 256, 384, 128),
    (2, 2, 300, 200, 64), (1, 2, 129, 1000, 128), (3, 1, 640, 130, 64)])
@pytest.mark.parametrize('dtype', ['bf16', 'f16'])
def test_matches_oracle(shape, dtype):
    q, k, v, scale = _inputs(*shape, dtype, seed=sum(shape))
    _check(_run(q, k, v, scale), q, k, v, scale, None, dtype)


def test_auto_selects_tc_for_long_sequences():
    q, k, v, scale = _inputs(1, 1, 256, 256, 128, 'bf16', 1)
    assert vectra_b200.kernel_for(q, k, v, scale) == 'tc'


@pytest.mark.parametrize('dtype', ['bf16', 'f16'])
def test_padding_bias_and_fully_masked_rows(dtype):
    B, H, nq, nk, D = 3, 2, 256, 384, 128
    q, k, v, scale = _inputs(B, H, nq, nk, D, dtype, 5)
    bias = torch.zeros(B, 1, 1, nk)
    bias[0, ..., 200:] = float('-inf')        # padded tail
    bias[1, ..., :] = float('-inf')           # every key masked -> NaN
    bias[1, ..., 7] = 0.0                     # ... except key 7
    bias[2, ..., ::3] = float('-inf')         # scattered mask
    out = _run(q, k, v, scale, bias.to(helpers.TORCH_DTYPES[dtype]))
    _check(out, q, k, v, scale, bias, dtype)
    # Batch row 1 attends to key 7 only: every query returns v[..., 7, :].
    np.testing.assert_allclose(
        out[1].float().cpu().numpy(),
        v[1, :, 7:8, :].float().expand(H, nq, D).numpy(), rtol=1e-2,
        atol=1e-3)
    full = torch.full((1, 1, 1, nk), float('-inf'))
    out_nan = _run(q[:1], k[:1], v[:1], scale, full)
    assert torch.isnan(out_nan.float()).all()


@pytest.mark.parametrize('spread', [4.0, 12.0])
def test_far_points_rescale_lazily(spread):
    # Large distances make the running max jump between tiles, which
    # exercises the O rescaling in TMEM.
    q, k, v, scale = _inputs(1, 2, 256, 1024, 128, 'bf16', 9, spread)
    scale = scale * 20
    _check(_run(q, k, v, scale), q, k, v, scale, None, 'bf16')


@pytest.mark.parametrize('s', [0.0, -0.01, 3.0])
def test_degenerate_and_negative_scales(s):
    q, k, v, _ = _inputs(1, 2, 128, 256, 64, 'bf16', 10)
    scale = torch.tensor(s)
    _check(_run(q, k, v, scale), q, k, v, scale, None, 'bf16')


def test_head_transposed_views():
    # q, k, v as views of one [B, N, 3*H*D] projection, as in the model.
    B, N, H, D = 2, 384, 4, 64
    gen = torch.Generator().manual_seed(11)
    proj = (torch.randn(B, N, 3 * H * D, generator=gen) / 8).bfloat16()
    q, k, v = (t.view(B, N, H, D).transpose(1, 2)
               for t in proj.cuda().split(H * D, dim=-1))
    assert not q.is_contiguous()
    scale = torch.full((1, H, 1, 1), 0.05)
    out = _run(q, k, v, scale)
    _check(out, q.cpu(), k.cpu(), v.cpu(), scale, None, 'bf16')


def test_deterministic_and_batch_slice_consistent():
    q, k, v, scale = _inputs(4, 2, 256, 256, 128, 'bf16', 12)
    args = [t.cuda() for t in (q, k, v, scale)]
    a = vectra_b200.rbf_attention(*args)
    assert torch.equal(a, vectra_b200.rbf_attention(*args))
    part = vectra_b200.rbf_attention(args[0][2:], args[1][2:], args[2][2:],
                                     args[3])
    assert torch.equal(part, a[2:])


def test_no_device_errors_after_tc_runs():
    from vectra_b200 import _lib  # pylint: disable=import-outside-toplevel
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.check_device_errors(stream) == _lib.OK
