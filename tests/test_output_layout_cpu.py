"""The operator's output layout rule (vectra_b200.custom_ops.output_strides)
and its fake implementation, without a GPU: a head-split view of a
[B, N, H * D] projection gets a head-transposed view of [B, N, H, Dv] memory
(so `.transpose(1, 2).reshape(B, N, H * Dv)` is a view); anything else a
contiguous output."""

import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from vectra_b200 import custom_ops


def test_projection_views_get_a_head_transposed_output():
    qkv = torch.empty(2, 7, 3, 4, 16)
    q, _, v = qkv.permute(2, 0, 3, 1, 4)
    st = custom_ops.output_strides(q, 8)
    assert st == (7 * 4 * 8, 8, 4 * 8, 1)
    out = torch.empty_strided((2, 4, 7, 8), st)
    assert out.transpose(1, 2).is_contiguous()
    del v


def test_other_layouts_get_a_contiguous_output():
    for q in (torch.empty(2, 4, 7, 16),              # contiguous
              torch.empty(2, 1, 7, 16),              # one head
              torch.empty(2, 7, 4, 16).transpose(1, 2)[:, :, :1],  # Nq = 1
              torch.empty(2, 4, 16, 7).transpose(2, 3)):  # D outermost
        assert custom_ops.output_strides(q, 8) == (
            q.shape[1] * q.shape[2] * 8, q.shape[2] * 8, 8, 1)


def test_fake_implementation_uses_the_rule():
    with FakeTensorMode():
        qkv = torch.empty(2, 7, 3, 4, 16, device='cuda')
        q, k, v = qkv.permute(2, 0, 3, 1, 4)
        scale = torch.ones(1, 4, 1, 1, device='cuda')
        out = torch.ops.vectra.rbf_attention(q, k, v, scale, None)
        assert out.shape == (2, 4, 7, 16)
        assert out.stride() == custom_ops.output_strides(q, 16)
        flat = torch.ops.vectra.rbf_attention(q.contiguous(), k, v, scale)
        assert flat.is_contiguous()
