"""The serving helpers' host logic on the CPU: the chunk split and the
padding rule of the reference's serving loop
(models/export/compile_entry.py:286-303)."""

import pytest
import torch

from vectra_b200 import serving


@pytest.mark.parametrize('n,b', [(1, 1), (1, 64), (63, 64), (64, 64),
                                 (65, 64), (1000, 64), (7, 3)])
def test_chunks_follow_the_reference_split(n, b):
    got = serving.chunks(n, b)
    assert got == [(s, min(s + b, n)) for s in range(0, n, b)]
    assert got[0][0] == 0 and got[-1][1] == n
    assert all(0 < stop - start <= b for start, stop in got)


@pytest.mark.parametrize('n,b', [(0, 4), (-1, 4), (4, 0)])
def test_chunks_reject_empty_batches_and_sizes(n, b):
    with pytest.raises(ValueError):
        serving.chunks(n, b)


def test_padding_repeats_the_last_request():
    chunk = torch.arange(12.).view(3, 2, 2)
    batch = torch.full((5, 2, 2), -1.0)
    batch[:3] = chunk
    assert serving.pad_in_place(batch, 3) is batch
    want = torch.cat([chunk, chunk[-1:].expand(2, 2, 2)])  # the reference's
    assert torch.equal(batch, want)
    full = chunk.clone()
    assert torch.equal(serving.pad_in_place(full, 3), chunk)
    for bad in (0, 4):
        with pytest.raises(ValueError):
            serving.pad_in_place(full, bad)


def test_serving_needs_cuda_example_inputs():
    with pytest.raises(ValueError):
        serving.GraphServingModel(lambda x: x, [torch.zeros(4, 2)])
    with pytest.raises(ValueError):
        serving.GraphServingModel(lambda x: x, [])
