"""vectra_scan_l2_topk_noalloc: the L2 scan for callers that cannot allocate
device memory (an FFI host handed device pointers with no CUDA allocator of
its own, or a serving loop that forbids cudaMalloc after start-up). Its
scratch is a static device array of the library; the caller passes only
inputs and outputs.

Called through the C ABI, its results must equal vectra_scan_l2_topk's with
a caller workspace bit for bit (the same kernels run) on calls in a row,
calls issued on different streams must not share the scratch at the same
time, and a scan needing more scratch than the array holds is refused with
VECTRA_ERR_UNSUPPORTED. This file is collected last and also passes alone.
"""

import numpy as np
import pytest
import torch

from vectra_b200 import _lib
from vectra_b200 import scan


def _inputs(nq, n, d, seed):
    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((n, d)).astype(np.float32)
    queries = (rows[rng.integers(0, n, nq)] +
               0.3 * rng.standard_normal((nq, d))).astype(np.float32)
    return torch.from_numpy(queries).cuda(), torch.from_numpy(rows).cuda()


def _same(a, b):
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_null_arguments_need_no_gpu():
    assert _lib.LIB.vectra_scan_l2_topk_noalloc(None, None) == _lib.ERR_NULL
    a = scan.L2Args()
    a.k = scan.MAX_K + 1
    assert _lib.LIB.vectra_scan_l2_topk_noalloc(a, None) == \
        _lib.ERR_UNSUPPORTED


@pytest.mark.gpu
@pytest.mark.parametrize('nq,n,d,k', [(1, 10, 16, 64), (8, 200000, 128, 64),
                                      (11, 20000, 64, 256), (5, 6000, 129, 33)])
def test_equals_the_workspace_entry_point(nq, n, d, k):
    queries, rows = _inputs(nq, n, d, seed=nq * 100 + k)
    other = (queries.flip(0) + 0.5).contiguous()
    # Two calls in a row: the second must not see the first one's scratch.
    first = scan.l2_topk_noalloc(queries, rows, k)
    second = scan.l2_topk_noalloc(other, rows, k)
    _same(first, scan.l2_topk(queries, rows, k))
    _same(second, scan.l2_topk(other, rows, k))


@pytest.mark.gpu
def test_candidate_lists():
    queries, rows = _inputs(6, 30000, 32, seed=3)
    rng = np.random.default_rng(4)
    cands = [np.sort(rng.choice(30000, size=size, replace=False))
             for size in (0, 5, 400, 9000, 15000, 30000)]
    _same(scan.l2_topk_noalloc(queries, rows, 40, cands),
          scan.l2_topk(queries, rows, 40, cands))


@pytest.mark.gpu
def test_calls_on_two_streams_take_turns_with_the_scratch():
    queries, rows = _inputs(16, 400000, 64, seed=5)
    want = [scan.l2_topk(queries[i::2].contiguous(), rows, 64)
            for i in range(2)]
    parts = [queries[i::2].contiguous() for i in range(2)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for _ in range(3):
        got = []
        for s, part in zip(streams, parts):
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):  # no ordering between the two streams
                got.append(scan.l2_topk_noalloc(part, rows, 64))
        for s in streams:
            torch.cuda.current_stream().wait_stream(s)
        for g, w in zip(got, want):
            _same(g, w)


@pytest.mark.gpu
def test_scans_beyond_the_static_scratch_are_refused():
    queries, rows = _inputs(64, 1 << 20, 16, seed=6)
    assert scan.workspace_bytes(64, 1 << 20, 64) > scan.NOALLOC_SCRATCH_BYTES
    with pytest.raises(scan.ScanError, match='unsupported'):
        scan.l2_topk_noalloc(queries, rows, 64)
    # The most queries (of 32 at most) whose scan fits the scratch.
    fit = max(nq for nq in (1, 2, 4, 8, 16, 32)
              if scan.workspace_bytes(nq, 1 << 20, 64) <=
              scan.NOALLOC_SCRATCH_BYTES)
    part = queries[:fit].contiguous()
    _same(scan.l2_topk_noalloc(part, rows, 64), scan.l2_topk(part, rows, 64))
