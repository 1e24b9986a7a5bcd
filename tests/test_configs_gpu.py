"""benchmark configs 1-4 and the config-5 attention site at their full sizes
(B200 only).

The oracle cannot finish a full batch quickly, so each config is checked
on seeded batch rows against the eager fp32 oracle (the acceptance gate), and
on the whole output through size-independent properties:
* every output row is a convex combination of the unmasked value rows, so
  each coordinate lies within their per-coordinate min and max;
* processing a slice of the batch reproduces the full run bit for bit
  (the multi-GPU harness relies on it).
"""

import numpy as np
import pytest
import torch

import vectra_b200
from oracle import rbf_oracle
from tests import helpers
from vectra_b200 import workloads

pytestmark = pytest.mark.gpu


def _oracle_rows(inp, rows, dtype):
    host = [None if t is None else t.float().cpu().numpy() for t in
            (inp.q, inp.k, inp.v, inp.scale, inp.key_bias)]
    q, k, v, s, b = rbf_oracle.sample_planes(*host, rows)
    return q, k, v, s, b


def _convexity(out, v, bias):
    v = v.float()
    if bias is not None:
        masked = torch.isinf(bias.float()).expand(v.shape[0], v.shape[1], 1,
                                                  v.shape[2])
        masked = masked.transpose(-1, -2)
        vmax = v.masked_fill(masked, -float('inf')).amax(-2, keepdim=True)
        vmin = v.masked_fill(masked, float('inf')).amin(-2, keepdim=True)
    else:
        vmax = v.amax(-2, keepdim=True)
        vmin = v.amin(-2, keepdim=True)
    o = out.float()
    slack = 1e-2 * (vmax - vmin).abs() + 1e-6
    assert bool(((o <= vmax + slack) & (o >= vmin - slack)).all())


@pytest.mark.parametrize('config', [1, 2, 3, 5])
def test_serving_configs_full_size(config):
    inp = workloads.make(config, device='cuda', seed=0)
    out = vectra_b200.rbf_attention(inp.q, inp.k, inp.v, inp.scale,
                                    inp.key_bias)
    torch.cuda.synchronize()
    assert out.shape == (*inp.q.shape[:3], inp.v.shape[3])
    assert torch.isfinite(out.float()).all()
    _convexity(out, inp.v, inp.key_bias)
    B = inp.q.shape[0]
    rows = np.unique(np.linspace(0, B - 1, 24).astype(int))
    q, k, v, s, b = _oracle_rows(inp, rows, inp.dtype)
    got = out[torch.as_tensor(rows).cuda()].double().cpu().numpy()
    helpers.check_eager_gate_tol(got, q, k, v, s, b, inp.dtype)
    helpers.check_reference_tol(got, q, k, v, s, b, inp.dtype)
    half = B // 2
    part = vectra_b200.rbf_attention(
        inp.q[half:], inp.k[half:], inp.v[half:], inp.scale,
        None if inp.key_bias is None else inp.key_bias[half:])
    assert torch.equal(part, out[half:])


def test_config4_long_sequence_planes():
    # The tensor-core config (B=16, H=16, L=4096, D=128) checked on a
    # batch slice; the oracle evaluates a few query rows of each plane.
    inp = workloads.make(4, device='cuda', seed=0, batch=1)
    out = vectra_b200.rbf_attention(inp.q, inp.k, inp.v, inp.scale)
    torch.cuda.synchronize()
    rows = np.array([0, 1, 777, 2048, 4095])
    q = inp.q[:, :, rows].float().cpu().numpy()
    k, v = (t.float().cpu().numpy() for t in (inp.k, inp.v))
    s = inp.scale.float().cpu().numpy()
    want = rbf_oracle.eager_rbf_attention(q, k, v, s)
    got = out[:, :, rows].double().cpu().numpy()
    rtol, atol = helpers.EAGER_GATE_TOL['bf16']
    helpers.assert_close(got, want, rtol, atol * float(np.abs(v).max()))
