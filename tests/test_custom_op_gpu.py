"""vectra::rbf_attention is a well-formed PyTorch operator on CUDA.

Mirrors kernels/tests/test_custom_op.py:37-82 on the GPU: opcheck (schema,
fake tensor, AOT dispatch static/dynamic), the fake implementation, and the
proof that the CUDA dispatch runs this library's kernels (its launch
counter moves) rather than any fallback.
"""

import pytest
import torch

import vectra_b200
from oracle import rbf_oracle
from tests import helpers

pytestmark = pytest.mark.gpu


def _inputs(dtype=torch.float32, bias=True, n_q=5):
    gen = torch.Generator().manual_seed(0)
    q = torch.randn(2, 3, n_q, 16, generator=gen)
    k = torch.randn(2, 3, 9, 16, generator=gen)
    v = torch.randn(2, 3, 9, 8, generator=gen)
    scale = torch.rand(1, 3, 1, 1, generator=gen) * 0.1 + 0.02
    key_bias = torch.zeros(2, 1, 1, 9)
    key_bias[1, ..., 7:] = float('-inf')
    args = [t.to('cuda', dtype) for t in (q, k, v)]
    args += [scale.cuda(), key_bias.to('cuda', dtype) if bias else None]
    return tuple(args)


@pytest.mark.parametrize('bias', [True, False])
@pytest.mark.parametrize('n_q', [1, 5])
def test_opcheck(bias, n_q):
    torch.library.opcheck(
        torch.ops.vectra.rbf_attention.default,
        _inputs(bias=bias, n_q=n_q),
        test_utils=('test_schema', 'test_faketensor',
                    'test_aot_dispatch_static', 'test_aot_dispatch_dynamic'))


def test_operator_matches_the_float64_oracle():
    args = _inputs()
    out = torch.ops.vectra.rbf_attention(*args)
    want = rbf_oracle.expanded_rbf_attention(
        *(t.cpu().numpy() for t in args))
    helpers.assert_close(out.double().cpu().numpy(), want, 1e-5, 1e-6)


def test_cuda_dispatch_launches_this_librarys_kernels():
    before = vectra_b200.launch_count()
    args = _inputs(dtype=torch.float16)
    out = torch.ops.vectra.rbf_attention(*args)
    torch.cuda.synchronize()
    assert vectra_b200.launch_count() == before + 1
    want = rbf_oracle.expanded_rbf_attention(
        *(t.float().cpu().numpy() for t in args))
    helpers.assert_close(out.double().cpu().numpy(), want, 1e-3, 1e-3)


def test_no_device_errors_after_the_suite_ran():
    from vectra_b200 import _lib  # pylint: disable=import-outside-toplevel
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.check_device_errors(stream) == _lib.OK


def test_runs_on_a_non_default_stream_and_device_guard():
    args = _inputs(dtype=torch.bfloat16, n_q=1)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        out = torch.ops.vectra.rbf_attention(*args)
    side.synchronize()
    want = rbf_oracle.expanded_rbf_attention(
        *(t.float().cpu().numpy() for t in args))
    helpers.assert_close(out.double().cpu().numpy(), want, 1e-2,
                         8e-3 * float(args[2].float().abs().max()))


def _projection_views(dtype=torch.bfloat16, B=3, N=11, H=4, D=32):
    """q, k, v as head-split views of one [B, N, 3 H D] projection (tokens
    outer to heads), like the compiled model's."""
    gen = torch.Generator().manual_seed(1)
    qkv = torch.randn(B, N, 3, H, D, generator=gen).to('cuda', dtype)
    q, k, v = qkv.permute(2, 0, 3, 1, 4)
    scale = torch.full((1, H, 1, 1), 0.05, device='cuda')
    return q, k, v, scale


@pytest.mark.parametrize('kernel', ['auto', 'generic', 'small', 'small_tc'])
def test_output_follows_the_projection_layout(kernel):
    from vectra_b200 import custom_ops  # pylint: disable=import-outside-toplevel
    q, k, v, scale = _projection_views()
    out = custom_ops.rbf_attention_with_kernel(q, k, v, scale, None, kernel)
    assert out.stride() == custom_ops.output_strides(q, v.shape[-1])
    assert out.transpose(1, 2).is_contiguous()  # the model's reshape: a view
    want = rbf_oracle.expanded_rbf_attention(
        *(t.float().cpu().numpy() for t in (q, k, v, scale)), None)
    helpers.assert_close(out.double().cpu().numpy(), want, 2e-2, 2e-2)
    contiguous = custom_ops.rbf_attention_with_kernel(
        q.contiguous(), k.contiguous(), v.contiguous(), scale, None, kernel)
    assert contiguous.is_contiguous()
    assert torch.equal(out, contiguous)  # same values, other layout


def test_opcheck_projection_views():
    torch.library.opcheck(
        torch.ops.vectra.rbf_attention.default, _projection_views(),
        test_utils=('test_schema', 'test_faketensor',
                    'test_aot_dispatch_static', 'test_aot_dispatch_dynamic'))
