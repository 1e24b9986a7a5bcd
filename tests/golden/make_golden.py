"""Generates the golden vectors that pin the oracle to the reference.

Run in a container that has the reference checkout (it imports the
reference's own `vectra_kernels.reference`, kernels/vectra_kernels/
reference.py:46-161, on the CPU):

    python tests/golden/make_golden.py --reference <checkout>/kernels

For each case it draws seeded inputs exactly as the reference's tests do
(torch.Generator().manual_seed(...) + torch.randn / torch.rand;
kernels/tests/test_parity.py:48-63, kernels/tests/test_edges.py), runs the
reference's four formulations and stores inputs and outputs in
tests/golden/<case>.npz:

* q, k, v: the inputs in their own width (float32; float16; bfloat16 as
  uint16 bit patterns), scale and bias as float32; `bias` is absent when
  the case has none;
* expanded: reference.expanded_rbf_attention (float64);
* eager: reference.eager_rbf_attention on float32 copies of the inputs;
* matmul: reference.matmul_rbf_attention (result in v's dtype, stored like
  the inputs);
* tiled: reference.tiled_rbf_attention (result in v's dtype, likewise);
* meta: JSON with the dtype, the seed and the reference file it came from.

The committed vectors are the reference's outputs; nothing on the GPU box
needs the reference checkout.
"""

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
DTYPES = {'f32': 'float32', 'f16': 'float16', 'bf16': 'bfloat16'}


def _cases(torch):
    """Yields (name, dtype, q, k, v, scale, bias, seed-description)."""
    td = {k: getattr(torch, v) for k, v in DTYPES.items()}

    # benchmark config 1: B=8, H=4, Lq=1, Lk=16, D=32, fp32, N(0,1),
    # gamma ~ U(0.05, 0.5) per head, no mask.
    gen = torch.Generator().manual_seed(0)
    q = torch.randn(8, 4, 1, 32, generator=gen)
    k = torch.randn(8, 4, 16, 32, generator=gen)
    v = torch.randn(8, 4, 16, 32, generator=gen)
    scale = 0.05 + 0.45 * torch.rand(1, 4, 1, 1, generator=gen)
    yield 'config1', 'f32', q, k, v, scale, None

    # kernels/tests/test_parity.py:48-63 `_inputs` at seed 0, with and
    # without the half-masked bias, for every dtype. The first shape is the
    # reference's (8,8,65,65,32,32) cut to one batch row and four heads,
    # the last (4,2,33,129,64,32) cut to one batch row (the GPU tests run
    # the full shapes against the oracle).
    shapes = {
        'p65': (1, 4, 65, 65, 32, 32),
        'p16': (1, 1, 16, 16, 16, 16),
        'p33x129': (1, 2, 33, 129, 64, 32),
    }
    for sname, shape in shapes.items():
        for dname in ('f32', 'f16', 'bf16'):
            for with_bias in (False, True):
                batch, heads, n_q, n_k, dim, value_dim = shape
                gen = torch.Generator().manual_seed(0)
                q = torch.randn(batch, heads, n_q, dim, generator=gen)
                k = torch.randn(batch, heads, n_k, dim, generator=gen)
                v = torch.randn(batch, heads, n_k, value_dim, generator=gen)
                scale = 1.0 / (2.0 * dim * (
                    0.5 + torch.rand(1, heads, 1, 1, generator=gen)))
                bias = None
                if with_bias:
                    bias = torch.zeros(batch, 1, 1, n_k)
                    bias[:, :, :, n_k // 2 + 1:] = float('-inf')
                yield (f'parity_{sname}_{dname}_{"bias" if with_bias else "nobias"}',
                       dname, q.to(td[dname]), k.to(td[dname]),
                       v.to(td[dname]), scale, bias)

    # kernels/tests/test_edges.py:37-46 tails.
    for n_q, n_k in [(1, 1), (1, 65), (17, 3), (63, 65), (65, 63), (129, 1),
                     (130, 200)]:
        gen = torch.Generator().manual_seed(n_q * 1000 + n_k)
        q = torch.randn(2, 3, n_q, 32, generator=gen)
        k = torch.randn(2, 3, n_k, 32, generator=gen)
        v = torch.randn(2, 3, n_k, 32, generator=gen)
        if n_q * n_k > 5000:  # Keep the fixture small: first batch row.
            q, k, v = q[:1], k[:1], v[:1]
        yield f'tail_{n_q}x{n_k}', 'f32', q, k, v, torch.tensor(0.02), None

    # test_edges.py:49-57 head widths.
    for dim, value_dim in [(8, 8), (48, 48), (80, 24), (100, 128), (128, 7)]:
        gen = torch.Generator().manual_seed(dim)
        q = torch.randn(1, 2, 40, dim, generator=gen)
        k = torch.randn(1, 2, 70, dim, generator=gen)
        v = torch.randn(1, 2, 70, value_dim, generator=gen)
        yield (f'dims_{dim}x{value_dim}', 'f32', q, k, v,
               torch.tensor(1.0 / (4.0 * dim)), None)

    # test_edges.py:60-71 all but one key masked.
    gen = torch.Generator().manual_seed(5)
    q = torch.randn(3, 2, 9, 16, generator=gen)
    k = torch.randn(3, 2, 70, 16, generator=gen)
    v = torch.randn(3, 2, 70, 16, generator=gen)
    bias = torch.full((3, 1, 1, 70), float('-inf'))
    bias[..., 0] = 0.0
    yield 'all_but_one', 'f32', q, k, v, torch.tensor(0.05), bias

    # test_edges.py:74-81 every key masked (NaN rows).
    gen = torch.Generator().manual_seed(9)
    q = torch.randn(1, 1, 4, 16, generator=gen)
    k = torch.randn(1, 1, 20, 16, generator=gen)
    v = torch.randn(1, 1, 20, 16, generator=gen)
    bias = torch.full((1, 1, 1, 20), float('-inf'))
    yield 'fully_masked', 'f32', q, k, v, torch.tensor(0.1), bias

    # test_edges.py:84-91 far points.
    gen = torch.Generator().manual_seed(6)
    q = torch.randn(2, 2, 10, 32, generator=gen) * 20
    k = torch.randn(2, 2, 50, 32, generator=gen) * 20
    v = torch.randn(2, 2, 50, 32, generator=gen)
    yield 'far', 'f32', q, k, v, torch.tensor(0.1), None

    # test_edges.py:94-100 degenerate and negative scales.
    for name, s in (('zero', 0.0), ('neg', -0.01), ('three', 3.0)):
        gen = torch.Generator().manual_seed(7)
        q = torch.randn(1, 2, 12, 16, generator=gen)
        k = torch.randn(1, 2, 30, 16, generator=gen)
        v = torch.randn(1, 2, 30, 16, generator=gen)
        yield f'scale_{name}', 'f32', q, k, v, torch.tensor(s), None

    # test_edges.py:103-114 head-transposed views and a per-head bias. The
    # stored q/k/v are contiguous copies; the GPU tests rebuild the views.
    gen = torch.Generator().manual_seed(8)
    projected = torch.randn(4, 65, 3 * 4 * 32, generator=gen)
    q, k, v = (t.view(4, 65, 4, 32).transpose(1, 2)
               for t in projected.split(4 * 32, dim=-1))
    bias = torch.zeros(4, 4, 1, 65)
    bias[1, 2, 0, 40:] = float('-inf')
    yield ('strided_per_head_bias', 'f32', q.contiguous(), k.contiguous(),
           v.contiguous(), torch.full((1, 4, 1, 1), 0.02), bias)

    # benchmark config 2 (serving), batch cut to 4: bf16, N(0,1)/sqrt(64),
    # gamma ~ U(0.1, 1.0), no mask.
    gen = torch.Generator().manual_seed(2)
    q = torch.randn(4, 8, 1, 64, generator=gen) / 8.0
    k = torch.randn(4, 8, 64, 64, generator=gen) / 8.0
    v = torch.randn(4, 8, 64, 64, generator=gen) / 8.0
    scale = 0.1 + 0.9 * torch.rand(1, 8, 1, 1, generator=gen)
    yield ('config2_b4', 'bf16', q.bfloat16(), k.bfloat16(), v.bfloat16(),
           scale, None)

    # benchmark config 3 (variable comparables), batch cut to 3: clustered
    # keys, prefix mask of length U{8..128} as a 0/-inf bf16 bias.
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(3, 8, 1, 64, generator=gen)
    centres = torch.randn(3, 8, 1, 64, generator=gen)
    k = centres + 0.1 * torch.randn(3, 8, 128, 64, generator=gen)
    v = torch.randn(3, 8, 128, 64, generator=gen) / 8.0
    scale = 0.1 + 1.9 * torch.rand(1, 8, 1, 1, generator=gen)
    lengths = torch.randint(8, 129, (3,), generator=gen)
    valid = torch.arange(128)[None, :] < lengths[:, None]
    bias = torch.zeros(3, 128).masked_fill(~valid, float('-inf'))
    yield ('config3_b3', 'bf16', q.bfloat16(), k.bfloat16(), v.bfloat16(),
           scale, bias.bfloat16()[:, None, None, :])


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument('--reference', required=True,
                        help='path to the reference kernels/ directory')
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    import torch  # pylint: disable=import-outside-toplevel
    from vectra_kernels import reference  # pylint: disable=import-outside-toplevel

    index = {}
    for name, dname, q, k, v, scale, bias in _cases(torch):
        f32 = [t.float() for t in (q, k, v)]

        def store(t):
            if t.dtype == torch.bfloat16:
                return t.view(torch.int16).numpy().view(np.uint16)
            return t.numpy()

        expanded = reference.expanded_rbf_attention(q, k, v, scale, bias)
        eager = reference.eager_rbf_attention(
            *f32, scale.float(), None if bias is None else bias.float())
        matmul = reference.matmul_rbf_attention(q, k, v, scale, bias)
        tiled = reference.tiled_rbf_attention(q, k, v, scale, bias)
        arrays = {
            'q': store(q), 'k': store(k), 'v': store(v),
            'scale': scale.float().numpy(),
            'expanded': expanded.numpy(),
            'eager': eager.numpy(),
            'matmul': store(matmul),
            'tiled': store(tiled),
        }
        if bias is not None:
            arrays['bias'] = bias.float().numpy()
        meta = {'dtype': dname,
                'source': 'kernels/vectra_kernels/reference.py:46-161',
                'torch': torch.__version__}
        arrays['meta'] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
        np.savez_compressed(os.path.join(HERE, f'{name}.npz'), **arrays)
        index[name] = dname
    with open(os.path.join(HERE, 'index.json'), 'w', encoding='utf-8') as f:
        json.dump(index, f, indent=1, sort_keys=True)
    print(f'wrote {len(index)} cases')


if __name__ == '__main__':
    main()
