"""The scan kernels (vectra_b200.scan) against the reference engine's own
results (tests/golden/scan_golden.npz) and the oracle pinned to them.

* PQ scans sum table entries in PqAdcDistance's order, and the tables
  kernel follows L2SquaredDistance's order as written: distances, nodes
  and tables are bit-identical to the reference's.
* The L2 scan forms sum_d (q_d - r_d)^2 in another order than the
  reference's sixteen lanes, so distances are held to the reference's own
  tolerance, 1e-5 (1 + d) (1 + |ref|) (engine/tests/unit/
  simd_parity_test.cc:22-26); the ranked nodes must match except where two
  candidates' distances are within that tolerance of each other.
"""

import os

import numpy as np
import pytest
import torch

from oracle import scan_oracle
from vectra_b200 import scan

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = np.load(os.path.join(ROOT, 'tests', 'golden', 'scan_golden.npz'))


def _tol(d, ref):
    return 1e-5 * (1.0 + d) * (1.0 + np.abs(ref))


def _check_l2(got_d, got_n, count, want_d, want_n, query, rows, d):
    """Sorted distances within tolerance; nodes equal up to near-ties; each
    returned distance is its node's distance."""
    k = want_d.shape[0]
    assert count == k
    gd = got_d[:k].astype(np.float64)
    gn = got_n[:k].astype(np.int64)
    assert np.all(np.diff(gd) >= 0)
    assert np.all(np.abs(gd - want_d) <= _tol(d, want_d))
    true_d = scan_oracle.l2_squared(query, rows[gn])
    assert np.all(np.abs(gd - true_d) <= _tol(d, true_d))
    kth = want_d[-1]
    firm = want_d < kth - _tol(d, kth)  # not near the boundary
    assert set(want_n[firm]) <= set(gn), 'a clearly nearer node is missing'
    mismatch = gn != want_n
    if mismatch.any():  # only near-ties may swap places
        assert np.all(np.abs(want_d[mismatch] - gd[mismatch]) <=
                      2 * _tol(d, want_d[mismatch]))


@pytest.mark.parametrize('case', sorted({k.split('/')[0] for k in GOLDEN.files
                                         if k.startswith('l2_')}))
def test_l2_matches_the_reference(case):
    rows = GOLDEN[f'{case}/rows']
    queries = GOLDEN[f'{case}/queries']
    k = GOLDEN[f'{case}/dist0'].shape[0]
    d = rows.shape[1]
    with_ids = f'{case}/ids0' in GOLDEN.files
    cands = ([GOLDEN[f'{case}/ids{i}'].astype(np.int64)
              for i in range(queries.shape[0])] if with_ids else None)
    gd, gn, gc = scan.l2_topk(torch.from_numpy(queries).cuda(),
                              torch.from_numpy(rows).cuda(), k, cands)
    gd, gn, gc = gd.cpu().numpy(), gn.cpu().numpy(), gc.cpu().numpy()
    for qi in range(queries.shape[0]):
        _check_l2(gd[qi], gn[qi], gc[qi], GOLDEN[f'{case}/dist{qi}'],
                  GOLDEN[f'{case}/nodes{qi}'], queries[qi], rows, d)


@pytest.mark.parametrize('case', sorted({k.split('/')[0] for k in GOLDEN.files
                                         if k.startswith('pq_')}))
def test_pq_matches_the_reference_bit_for_bit(case):
    query = torch.from_numpy(GOLDEN[f'{case}/query']).cuda()[None]
    codebooks = torch.from_numpy(GOLDEN[f'{case}/codebooks']).cuda()
    m = codebooks.shape[0]
    table = scan.pq_distance_tables(query, codebooks, m)
    np.testing.assert_array_equal(table[0].cpu().numpy(),
                                  GOLDEN[f'{case}/table'])
    k = GOLDEN[f'{case}/dist'].shape[0]
    gd, gn, gc = scan.pq_topk(table, torch.from_numpy(
        GOLDEN[f'{case}/codes']).cuda(), k)
    assert int(gc[0]) == k
    np.testing.assert_array_equal(gd[0].cpu().numpy(), GOLDEN[f'{case}/dist'])
    np.testing.assert_array_equal(gn[0].cpu().numpy().astype(np.int64),
                                  GOLDEN[f'{case}/nodes'])


def _l2_random(nq, n, d, k, seed, lists=False):
    rng = np.random.default_rng(seed)
    rows = rng.standard_normal((n, d)).astype(np.float32)
    queries = (rows[rng.integers(0, n, nq)] +
               0.3 * rng.standard_normal((nq, d))).astype(np.float32)
    cands = None
    if lists:
        cands = [np.sort(rng.choice(n, size=int(rng.integers(0, n // 2 + 1)),
                                    replace=False)) for _ in range(nq)]
    gd, gn, gc = scan.l2_topk(torch.from_numpy(queries).cuda(),
                              torch.from_numpy(rows).cuda(), k, cands)
    gd, gn, gc = gd.cpu().numpy(), gn.cpu().numpy(), gc.cpu().numpy()
    for qi in range(nq):
        ids = None if cands is None else cands[qi]
        wd, wn = scan_oracle.exhaustive_l2_topk(queries[qi], rows, k, ids)
        cnt = wd.shape[0]
        assert gc[qi] == cnt
        assert np.all(gn[qi, cnt:] == -1) and np.all(np.isinf(gd[qi, cnt:]))
        if cnt:
            _check_l2(gd[qi], gn[qi], cnt, wd, wn, queries[qi], rows, d)


@pytest.mark.parametrize('k', [1, 10, 32, 33, 64, 65, 128, 200, 256])
def test_l2_every_list_width(k):
    _l2_random(11, 20000, 64, k, seed=k)


@pytest.mark.parametrize('d', [1, 3, 4, 17, 64, 128, 129, 768])
def test_l2_dimensions(d):
    _l2_random(9, 6000, d, 16, seed=d)


def test_l2_many_tiles_and_query_groups():
    _l2_random(37, 150000, 128, 64, seed=7)


def test_l2_per_query_candidate_lists():
    _l2_random(13, 30000, 32, 40, seed=8, lists=True)


def test_l2_fewer_rows_than_k():
    _l2_random(3, 10, 16, 64, seed=9)


def test_l2_strided_rows():
    rng = np.random.default_rng(10)
    base = torch.from_numpy(rng.standard_normal((5000, 80)).astype(
        np.float32)).cuda()
    rows = base[:, :64]  # row stride 80
    queries = base[:4, 8:72].contiguous()
    gd, gn, _ = scan.l2_topk(queries, rows, 20)
    for qi in range(4):
        wd, wn = scan_oracle.exhaustive_l2_topk(
            queries[qi].cpu().numpy(), rows.cpu().numpy(), 20)
        _check_l2(gd[qi].cpu().numpy(), gn[qi].cpu().numpy(), 20, wd, wn,
                  queries[qi].cpu().numpy(), rows.cpu().numpy(), 64)


@pytest.mark.parametrize('m,k', [(1, 5), (3, 17), (8, 64), (16, 100),
                                 (17, 33), (32, 256), (64, 64)])
def test_pq_random_bit_for_bit(m, k):
    rng = np.random.default_rng(m * 1000 + k)
    nq, n = 6, 30000
    tables = (rng.random((nq, m, 256)) * 3).astype(np.float32)
    codes = rng.integers(0, 256, (n, m), dtype=np.uint8)
    gd, gn, gc = scan.pq_topk(torch.from_numpy(tables).cuda(),
                              torch.from_numpy(codes).cuda(), k)
    for qi in range(nq):
        wd, wn = scan_oracle.pq_topk(tables[qi], codes, k)
        assert int(gc[qi]) == k
        np.testing.assert_array_equal(gd[qi].cpu().numpy(), wd)
        np.testing.assert_array_equal(gn[qi].cpu().numpy().astype(np.int64),
                                      wn)


def test_pq_candidate_lists_and_ties():
    rng = np.random.default_rng(11)
    m, n, nq, k = 8, 5000, 5, 30
    tables = np.floor(rng.random((nq, m, 256)) * 4).astype(np.float32)
    codes = rng.integers(0, 256, (n, m), dtype=np.uint8)  # many ties
    cands = [np.sort(rng.choice(n, size=size, replace=False))
             for size in (0, 7, 300, 2500, n)]
    gd, gn, gc = scan.pq_topk(torch.from_numpy(tables).cuda(),
                              torch.from_numpy(codes).cuda(), k, cands)
    for qi in range(nq):
        wd, wn = scan_oracle.pq_topk(tables[qi], codes, k, cands[qi])
        cnt = wd.shape[0]
        assert int(gc[qi]) == cnt
        np.testing.assert_array_equal(gd[qi, :cnt].cpu().numpy(), wd)
        np.testing.assert_array_equal(
            gn[qi, :cnt].cpu().numpy().astype(np.int64), wn)


@pytest.mark.parametrize('d,m', [(16, 16), (128, 16), (96, 8), (64, 64),
                                 (30, 3)])
def test_distance_tables_bit_for_bit(d, m):
    rng = np.random.default_rng(d + m)
    queries = rng.standard_normal((5, d)).astype(np.float32)
    codebooks = rng.standard_normal((m, 256, d // m)).astype(np.float32)
    got = scan.pq_distance_tables(torch.from_numpy(queries).cuda(),
                                  torch.from_numpy(codebooks).cuda(), m)
    np.testing.assert_array_equal(got.cpu().numpy(),
                                  scan_oracle.distance_tables(queries,
                                                              codebooks))


def test_results_are_deterministic_and_use_the_launching_stream():
    rng = np.random.default_rng(12)
    rows = torch.from_numpy(rng.standard_normal((40000, 64)).astype(
        np.float32)).cuda()
    queries = rows[:8] + 0.1
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        a = scan.l2_topk(queries, rows, 64)
    torch.cuda.current_stream().wait_stream(side)
    b = scan.l2_topk(queries, rows, 64)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


# Scans of more than 32,768 candidates run in levels: a sample's k-th
# distance bounds the next level, whose select keeps the k nearest of the
# few candidates under it; a last level that admits more than its buffer
# holds (mass ties) is redone by the warp-list scan. The cases below reach
# each of these.

def _pq_check(tables, codes, k, cands=None):
    gd, gn, gc = scan.pq_topk(torch.from_numpy(tables).cuda(),
                              torch.from_numpy(codes).cuda(), k, cands)
    for qi in range(tables.shape[0]):
        ids = None if cands is None else cands[qi]
        wd, wn = scan_oracle.pq_topk(tables[qi], codes, k, ids)
        cnt = wd.shape[0]
        assert int(gc[qi]) == cnt
        np.testing.assert_array_equal(gd[qi, :cnt].cpu().numpy(), wd)
        np.testing.assert_array_equal(
            gn[qi, :cnt].cpu().numpy().astype(np.int64), wn)
        assert np.all(gn[qi, cnt:].cpu().numpy() == -1)


def test_pq_three_levels_bit_for_bit():
    rng = np.random.default_rng(21)
    tables = (rng.random((3, 8, 256)) * 3).astype(np.float32)
    codes = rng.integers(0, 256, (1 << 20, 8), dtype=np.uint8)
    _pq_check(tables, codes, 256)  # k = 256 over 1M codes: three levels


def test_pq_ties_at_the_bound_across_levels():
    rng = np.random.default_rng(22)
    tables = np.floor(rng.random((4, 8, 256)) * 4).astype(np.float32)
    codes = rng.integers(0, 256, (200000, 8), dtype=np.uint8)
    _pq_check(tables, codes, 100)


def test_pq_mass_ties_overflow_and_rescan():
    codes = np.random.default_rng(23).integers(0, 256, (100000, 16),
                                               dtype=np.uint8)
    tables = np.ones((2, 16, 256), np.float32)  # every distance is 16
    tables[1, 3, :] = 0.5  # and 15.5 for the second query
    _pq_check(tables, codes, 50)


def test_l2_identical_rows_overflow_and_rescan():
    rows = np.tile(np.arange(16, dtype=np.float32), (60000, 1))
    queries = np.zeros((3, 16), np.float32)
    queries[1] = 1.0
    gd, gn, gc = scan.l2_topk(torch.from_numpy(queries).cuda(),
                              torch.from_numpy(rows).cuda(), 20)
    for qi in range(3):
        wd, wn = scan_oracle.exhaustive_l2_topk(queries[qi], rows, 20)
        assert int(gc[qi]) == 20
        np.testing.assert_array_equal(gn[qi].cpu().numpy().astype(np.int64),
                                      wn)  # nodes 0..19: ties by node id
        assert np.all(gd[qi].cpu().numpy() == gd[qi, 0].item())


def test_l2_candidate_lists_of_every_size():
    rng = np.random.default_rng(24)
    n, d = 150000, 32
    rows = rng.standard_normal((n, d)).astype(np.float32)
    queries = (rows[:5] + 0.2 * rng.standard_normal((5, d))).astype(
        np.float32)
    cands = [np.zeros(0, np.int64), np.array([4, 17, 3]),
             rng.choice(n, 40000, replace=False),
             rng.choice(n, 120000, replace=False), np.arange(n)]
    gd, gn, gc = scan.l2_topk(torch.from_numpy(queries).cuda(),
                              torch.from_numpy(rows).cuda(), 64, cands)
    gd, gn, gc = gd.cpu().numpy(), gn.cpu().numpy(), gc.cpu().numpy()
    for qi in range(5):
        wd, wn = scan_oracle.exhaustive_l2_topk(queries[qi], rows, 64,
                                                cands[qi])
        cnt = wd.shape[0]
        assert gc[qi] == cnt
        assert np.all(gn[qi, cnt:] == -1) and np.all(np.isinf(gd[qi, cnt:]))
        if cnt:
            _check_l2(gd[qi], gn[qi], cnt, wd, wn, queries[qi], rows, d)


def test_duplicate_candidate_ids_are_kept_like_the_reference_heap():
    # PushBounded (shard_index.cc:111-120) keeps the k smallest of the
    # multiset: a repeated id appears as often as it is among them.
    rng = np.random.default_rng(25)
    tables = np.repeat((rng.random((1, 8, 256)) * 3).astype(np.float32), 3,
                       axis=0)
    codes = rng.integers(0, 256, (50000, 8), dtype=np.uint8)
    best = int(np.argmin(scan_oracle.pq_adc(tables[0], codes)))
    lists = [np.concatenate([np.full(copies, best), rng.choice(50000, 500)])
             for copies in (7, 3000, 40000)]  # sorted, past the sort, re-scan
    _pq_check(tables, codes, 30, lists)


@pytest.mark.parametrize('nq,d', [(3, 256), (8, 64), (2, 192), (5, 128)])
def test_l2_bulk_copy_shapes(nq, d):
    # dim = 64 NC with aligned rows runs the bulk-copy level kernel (NC 1,
    # 2, 4); 192 (NC 3) runs the lane-per-row one.
    _l2_random(nq, 70000, d, 48, seed=d + nq)


def test_l2_bulk_copy_row_stride_and_tail():
    rng = np.random.default_rng(26)
    base = torch.from_numpy(rng.standard_normal((50001, 132)).astype(
        np.float32)).cuda()
    rows = base[:, :128]  # stride 132 floats, 50,001 rows (a ragged batch)
    queries = (base[7:11, :128] + 0.05).contiguous()
    gd, gn, gc = scan.l2_topk(queries, rows, 33)
    for qi in range(4):
        wd, wn = scan_oracle.exhaustive_l2_topk(
            queries[qi].cpu().numpy(), rows.cpu().numpy(), 33)
        _check_l2(gd[qi].cpu().numpy(), gn[qi].cpu().numpy(), 33, wd, wn,
                  queries[qi].cpu().numpy(), rows.cpu().numpy(), 128)


def test_l2_bulk_copy_suffix_column_view():
    # rows = base[:, 64:] of an [N, 128] tensor: stride 128, dimension 64,
    # and the last row's final element is the storage's last element. A
    # batch copy ends at its last row's final element, never a full stride
    # past it.
    rng = np.random.default_rng(31)
    n = 40003
    base = torch.from_numpy(rng.standard_normal((n, 128)).astype(
        np.float32)).cuda()
    rows = base[:, 64:]
    assert (rows.storage_offset() + (n - 1) * rows.stride(0) + 64 ==
            base.untyped_storage().nbytes() // 4)
    queries = (base[[5, 17, 30001], 64:] + 0.03).contiguous()
    gd, gn, _ = scan.l2_topk(queries, rows, 24)
    host_rows = rows.cpu().numpy()
    for qi in range(3):
        q = queries[qi].cpu().numpy()
        wd, wn = scan_oracle.exhaustive_l2_topk(q, host_rows, 24)
        _check_l2(gd[qi].cpu().numpy(), gn[qi].cpu().numpy(), 24, wd, wn,
                  q, host_rows, 64)


def test_l2_rows_with_a_large_common_offset():
    # Coordinates near 1,000 (e.g. unnormalised features): q_d - r_d of
    # nearby float32 values is exact, so direct differences keep the
    # reference's tolerance where ||q||^2 + ||r||^2 - 2 q.r would lose it.
    rng = np.random.default_rng(27)
    n, d = 60000, 128
    rows = (1000.0 + rng.standard_normal((n, d))).astype(np.float32)
    queries = (rows[rng.integers(0, n, 4)] +
               0.05 * rng.standard_normal((4, d))).astype(np.float32)
    gd, gn, gc = scan.l2_topk(torch.from_numpy(queries).cuda(),
                              torch.from_numpy(rows).cuda(), 32)
    gd, gn = gd.cpu().numpy(), gn.cpu().numpy()
    for qi in range(4):
        wd, wn = scan_oracle.exhaustive_l2_topk(queries[qi], rows, 32)
        _check_l2(gd[qi], gn[qi], 32, wd, wn, queries[qi], rows, d)
