"""Edge shapes, values and argument forms on the CUDA operator (B200 only).

Follows kernels/tests/test_edges.py (tails, head widths, masking, far
points, degenerate scales, strided views) and the argument forms the
compile pass emits (compiler/vectra_compiler/replacement.py:216-231: a 0-dim
float32 `scalar_tensor` scale, a reciprocal of a half-precision [1,H,1,1]
divisor, a bias in the block dtype), plus the error behaviour of the
reference's host wrapper (spatial_rbf_attention.py:220-225).
"""

import numpy as np
import pytest
import torch

import vectra_b200
from oracle import rbf_oracle
from tests import golden
from tests import helpers

pytestmark = pytest.mark.gpu


def _cuda(a, dtype=torch.float32):
    return torch.as_tensor(np.asarray(a, np.float32)).to('cuda', dtype)


def test_head_transposed_views_and_per_head_bias():
    # kernels/tests/test_edges.py:103-114: q, k, v are views of one
    # [B, N, 3*H*D] projection; nothing is copied.
    c = golden.load('strided_per_head_bias')
    B, H, N, D = c['q'].shape
    parts = [torch.as_tensor(c[n]).transpose(1, 2).reshape(B, N, H * D)
             for n in ('q', 'k', 'v')]
    projected = torch.cat(parts, dim=-1).cuda()
    q, k, v = (t.view(B, N, H, D).transpose(1, 2)
               for t in projected.split(H * D, dim=-1))
    assert not q.is_contiguous()
    out = vectra_b200.rbf_attention(q, k, v, _cuda(c['scale']),
                                    _cuda(c['bias']))
    helpers.assert_close(out.double().cpu().numpy(), c['expanded'],
                         1e-4, 1e-5)


@pytest.mark.parametrize('dtype', ['f32', 'bf16'])
def test_non_unit_inner_strides(dtype):
    q, k, v, scale, bias = helpers.parity_inputs((2, 3, 9, 20, 16, 16),
                                                 dtype, 4, True)
    td = helpers.TORCH_DTYPES[dtype]
    # Interleave with junk along D so the innermost stride is 2.
    def spread(a):
        t = _cuda(a, td)
        wide = torch.full((*t.shape[:-1], 2 * t.shape[-1]), 1e4, dtype=td,
                          device='cuda')
        wide[..., ::2] = t
        return wide[..., ::2]
    out = vectra_b200.rbf_attention(spread(q), spread(k), spread(v),
                                    _cuda(scale), _cuda(bias))
    helpers.check_reference_tol(out.double().cpu().numpy(), q, k, v, scale,
                                bias, dtype)


@pytest.mark.parametrize('kernel', ['auto', 'generic', 'decode'])
def test_all_but_one_candidate_masked(kernel):
    # test_edges.py:60-71 (with Nq == 1 so the decode kernel takes it too).
    gen = torch.Generator().manual_seed(5)
    q = torch.randn(3, 2, 1, 32, generator=gen)
    k = torch.randn(3, 2, 70, 32, generator=gen)
    v = torch.randn(3, 2, 70, 32, generator=gen)
    bias = torch.full((3, 1, 1, 70), float('-inf'))
    bias[..., 0] = 0.0
    out = helpers.run(q.numpy(), k.numpy(), v.numpy(), np.float32(0.05),
                      bias.numpy(), 'f32', kernel=kernel)
    np.testing.assert_allclose(out, v[:, :, :1, :].double().numpy(),
                               rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize('kernel', ['auto', 'generic', 'decode'])
@pytest.mark.parametrize('dtype', ['f32', 'bf16'])
def test_fully_masked_rows_are_nan(kernel, dtype):
    # test_edges.py:74-81: every key masked -> NaN, like eager softmax.
    gen = torch.Generator().manual_seed(9)
    q = torch.randn(2, 2, 1, 32, generator=gen).numpy()
    k = torch.randn(2, 2, 40, 32, generator=gen).numpy()
    v = torch.randn(2, 2, 40, 32, generator=gen).numpy()
    bias = np.full((2, 1, 1, 40), -np.inf, np.float32)
    bias[1, ..., 3] = 0.0  # batch row 1 keeps one key
    out = helpers.run(q, k, v, np.float32(0.1), bias, dtype, kernel=kernel)
    assert np.isnan(out[0]).all()
    assert np.isfinite(out[1]).all()


def test_bias_varying_across_queries_raises_value_error():
    q = torch.randn(1, 1, 4, 16, device='cuda')
    k = torch.randn(1, 1, 6, 16, device='cuda')
    bias = torch.zeros(1, 1, 4, 6, device='cuda')
    with pytest.raises(ValueError, match='constant across queries'):
        vectra_b200.rbf_attention(q, k, k, torch.tensor(0.1), bias)


def test_mismatched_dtypes_raise_value_error():
    q = torch.randn(1, 1, 4, 16, device='cuda')
    with pytest.raises(ValueError, match='share a dtype'):
        vectra_b200.rbf_attention(q, q.half(), q, torch.tensor(0.1))


def test_bad_shapes_raise_value_error():
    q = torch.randn(1, 2, 4, 16, device='cuda')
    k = torch.randn(1, 2, 6, 8, device='cuda')
    with pytest.raises(ValueError):
        vectra_b200.rbf_attention(q, k, k, torch.tensor(0.1))
    with pytest.raises(ValueError):
        vectra_b200.rbf_attention(q, q, q, torch.ones(1, 3, 1, 1,
                                                      device='cuda'))


def test_dispatch_by_device_never_crosses_it():
    # CPU tensors run the CPU implementation (no kernel launch); CUDA
    # tensors always launch this library's kernel; mixed devices raise.
    q = torch.randn(1, 1, 2, 8)
    before = vectra_b200.launch_count()
    out = torch.ops.vectra.rbf_attention(q, q, q, torch.tensor(0.1))
    assert out.device.type == 'cpu' and vectra_b200.launch_count() == before
    qc = q.cuda()
    got = torch.ops.vectra.rbf_attention(qc, qc, qc, torch.tensor(0.1))
    torch.cuda.synchronize()
    assert vectra_b200.launch_count() == before + 1
    torch.testing.assert_close(got.cpu(), out, rtol=1e-5, atol=1e-6)
    with pytest.raises((ValueError, RuntimeError)):
        torch.ops.vectra.rbf_attention(qc, q, qc, torch.tensor(0.1))


def test_forced_kernel_that_cannot_run_raises():
    q = torch.randn(1, 1, 4, 16, device='cuda')
    with pytest.raises(ValueError, match='forced kernel'):
        vectra_b200.rbf_attention_with_kernel(q, q, q, torch.tensor(0.1),
                                              kernel='decode')


@pytest.mark.parametrize('scale_form', [
    'cpu_scalar', 'cuda_scalar_f32', 'half_per_head', 'bf16_per_head',
    'double_per_head', 'per_batch_head', 'reciprocal_of_half_divisor'])
@pytest.mark.parametrize('nq', [1, 7])
def test_scale_argument_forms(scale_form, nq):
    B, H, nk, D = 3, 4, 33, 32
    gen = torch.Generator().manual_seed(11)
    q = torch.randn(B, H, nq, D, generator=gen)
    k = torch.randn(B, H, nk, D, generator=gen)
    v = torch.randn(B, H, nk, D, generator=gen)
    per_head = 0.01 + 0.04 * torch.rand(1, H, 1, 1, generator=gen)
    divisor = (1.0 / per_head).half()
    forms = {
        'cpu_scalar': torch.tensor(0.03),
        'cuda_scalar_f32': torch.scalar_tensor(0.03, dtype=torch.float32,
                                               device='cuda'),
        'half_per_head': per_head.half().cuda(),
        'bf16_per_head': per_head.bfloat16().cuda(),
        'double_per_head': per_head.double().cuda(),
        'per_batch_head': (0.01 + 0.04 * torch.rand(B, H, 1, 1,
                                                    generator=gen)).cuda(),
        'reciprocal_of_half_divisor': torch.reciprocal(divisor.cuda()),
    }
    scale = forms[scale_form]
    out = vectra_b200.rbf_attention(q.cuda(), k.cuda(), v.cuda(), scale)
    expected = rbf_oracle.expanded_rbf_attention(
        q.numpy(), k.numpy(), v.numpy(), scale.double().cpu().numpy())
    helpers.assert_close(out.double().cpu().numpy(), expected, 1e-4, 1e-5)


@pytest.mark.parametrize('bias_dtype', [torch.float32, torch.float16,
                                        torch.bfloat16, torch.float64])
@pytest.mark.parametrize('bias_shape', ['b11n', 'bh1n', 'n', '111n'])
@pytest.mark.parametrize('nq', [1, 5])
def test_bias_argument_forms(bias_dtype, bias_shape, nq):
    B, H, nk, D = 2, 4, 40, 64
    gen = torch.Generator().manual_seed(12)
    q = torch.randn(B, H, nq, D, generator=gen) / 8
    k = torch.randn(B, H, nk, D, generator=gen) / 8
    v = torch.randn(B, H, nk, D, generator=gen)
    full = torch.zeros(B, H, 1, nk)
    full[0, :, :, 30:] = float('-inf')
    full[1, 1, :, 5:9] = float('-inf')
    forms = {'b11n': full[:, :1], 'bh1n': full, 'n': full[0, 0, 0],
             '111n': full[:1, :1]}
    bias = forms[bias_shape]
    out = vectra_b200.rbf_attention(q.bfloat16().cuda(), k.bfloat16().cuda(),
                                    v.bfloat16().cuda(), torch.tensor(0.5),
                                    bias.to('cuda', bias_dtype))
    qn, kn, vn = (rbf_oracle.round_to(t.numpy(), 'bf16') for t in (q, k, v))
    bn = bias.to(bias_dtype).double().numpy()
    helpers.check_reference_tol(out.double().cpu().numpy(), qn, kn, vn,
                                np.float32(0.5), bn, 'bf16')


def test_no_keys_gives_zeros_and_empty_batches_work():
    q = torch.randn(2, 3, 4, 16, device='cuda')
    k = torch.empty(2, 3, 0, 16, device='cuda')
    out = vectra_b200.rbf_attention(q, k, k, torch.tensor(0.1))
    assert out.shape == (2, 3, 4, 16)
    assert (out == 0).all()  # softmax(empty) @ v = zeros, as eager
    q0 = torch.randn(0, 3, 1, 16, device='cuda')
    out0 = vectra_b200.rbf_attention(q0, q0, q0, torch.tensor(0.1))
    assert out0.shape == (0, 3, 1, 16)


@pytest.mark.parametrize('kernel', ['generic', 'decode'])
def test_deterministic_and_shard_consistent(kernel):
    # The multi-GPU harness slices the batch; a slice must reproduce the
    # full run's rows bit for bit, and repeated runs must agree.
    gen = torch.Generator().manual_seed(13)
    q = torch.randn(64, 8, 1, 64, generator=gen).bfloat16().cuda()
    k = torch.randn(64, 8, 64, 64, generator=gen).bfloat16().cuda()
    v = torch.randn(64, 8, 64, 64, generator=gen).bfloat16().cuda()
    s = torch.rand(1, 8, 1, 1, generator=gen).cuda()
    run = lambda a, b, c: vectra_b200.rbf_attention_with_kernel(  # noqa
        a, b, c, s, kernel=kernel)
    full = run(q, k, v)
    assert torch.equal(full, run(q, k, v))
    for lo, hi in ((0, 16), (16, 48), (48, 64)):
        assert torch.equal(full[lo:hi], run(q[lo:hi], k[lo:hi], v[lo:hi]))


def test_masked_key_contents_are_never_used():
    # Keys with a -inf bias carry zero weight; changing their rows (to large
    # finite junk) must not change a single output bit (the decode kernel
    # does not even fetch them).
    gen = torch.Generator().manual_seed(14)
    B, H, nk, D = 32, 8, 128, 64
    q = torch.randn(B, H, 1, D, generator=gen).bfloat16().cuda()
    k = torch.randn(B, H, nk, D, generator=gen).bfloat16().cuda()
    v = torch.randn(B, H, nk, D, generator=gen).bfloat16().cuda()
    lengths = torch.randint(1, nk + 1, (B,), generator=gen)
    valid = torch.arange(nk)[None] < lengths[:, None]
    bias = torch.zeros(B, nk).masked_fill(~valid, float('-inf'))
    bias = bias.bfloat16()[:, None, None, :].cuda()
    s = torch.rand(1, H, 1, 1, generator=gen).cuda()
    clean = vectra_b200.rbf_attention(q, k, v, s, bias)
    mask = (~valid).cuda()[:, None, :, None].expand(B, H, nk, D)
    k2 = k.masked_fill(mask, 300.0)
    v2 = v.masked_fill(mask, -300.0)
    assert torch.equal(clean, vectra_b200.rbf_attention(q, k2, v2, s, bias))
