"""The scan path on the CPU: the oracle pinned to the reference engine's own
code, the C ABI's exports and the wrapper's argument checks.

The oracle (oracle/scan_oracle.py) is checked bit for bit against
tests/golden/scan_golden.npz, outputs of the reference's own
simd_distance.cc / pq_codec.cc compiled by oracle/Makefile
(tests/golden/make_scan_golden.py), and, where oracle/_ref has been built
here, against that library directly on fresh random inputs
(engine/tests/unit/simd_parity_test.cc checks the same functions at every
dimension 1..300).
"""

import os
import re

import numpy as np
import pytest
import torch

from oracle import scan_oracle
from vectra_b200 import _lib
from vectra_b200 import scan

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = np.load(os.path.join(ROOT, 'tests', 'golden', 'scan_golden.npz'))
REF = scan_oracle.load_reference()
needs_ref = pytest.mark.skipif(REF is None,
                               reason='oracle/_ref not built (make -C oracle)')


def _cases(prefix):
    return sorted({k.split('/')[0] for k in GOLDEN.files
                   if k.startswith(prefix)})


@pytest.mark.parametrize('case', _cases('l2_'))
def test_oracle_l2_topk_matches_golden(case):
    rows, queries = GOLDEN[f'{case}/rows'], GOLDEN[f'{case}/queries']
    k = GOLDEN[f'{case}/dist0'].shape[0]
    for qi in range(queries.shape[0]):
        key = f'{case}/ids{qi}'
        ids = GOLDEN[key] if key in GOLDEN.files else None
        d, n = scan_oracle.exhaustive_l2_topk(queries[qi], rows, k, ids)
        np.testing.assert_array_equal(d, GOLDEN[f'{case}/dist{qi}'])
        np.testing.assert_array_equal(n, GOLDEN[f'{case}/nodes{qi}'])


@pytest.mark.parametrize('case', _cases('pq_'))
def test_oracle_pq_matches_golden(case):
    table = scan_oracle.distance_tables(GOLDEN[f'{case}/query'][None],
                                        GOLDEN[f'{case}/codebooks'])[0]
    np.testing.assert_array_equal(table, GOLDEN[f'{case}/table'])
    k = GOLDEN[f'{case}/dist'].shape[0]
    d, n = scan_oracle.pq_topk(table, GOLDEN[f'{case}/codes'], k)
    np.testing.assert_array_equal(d, GOLDEN[f'{case}/dist'])
    np.testing.assert_array_equal(n, GOLDEN[f'{case}/nodes'])


@needs_ref
def test_oracle_l2_matches_the_compiled_reference_at_every_dimension():
    rng = np.random.default_rng(1)
    for d in range(1, 301):
        q = rng.standard_normal(d).astype(np.float32)
        rows = rng.standard_normal((8, d)).astype(np.float32)
        np.testing.assert_array_equal(scan_oracle.l2_squared(q, rows),
                                      REF.l2_distances(q, rows))


@needs_ref
@pytest.mark.parametrize('m', [1, 2, 3, 4, 5, 8, 16, 17, 32, 64])
def test_oracle_pq_matches_the_compiled_reference(m):
    rng = np.random.default_rng(m)
    table = (rng.random((m, 256)) * 4).astype(np.float32)
    codes = rng.integers(0, 256, (64, m), dtype=np.uint8)
    want = np.array([REF.pq_adc(table, c) for c in codes], np.float32)
    np.testing.assert_array_equal(scan_oracle.pq_adc(table, codes), want)


@needs_ref
def test_oracle_topk_breaks_ties_by_node_like_the_reference():
    rows = np.zeros((50, 4), np.float32)  # every distance ties
    rows[7] = 5.0
    q = np.zeros(4, np.float32)
    for ids in (None, np.array([49, 3, 12, 0, 7, 30], np.uint32)):
        d0, n0 = REF.exhaustive_topk(q, rows, 5, ids)
        d1, n1 = scan_oracle.exhaustive_l2_topk(q, rows, 5, ids)
        np.testing.assert_array_equal(d0, d1)
        np.testing.assert_array_equal(n0, n1)


def test_library_exports_every_scan_function():
    text = open(os.path.join(ROOT, 'include', 'vectra_scan.h'),
                encoding='utf-8').read()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    declared = sorted(set(re.findall(r'\b(vectra_(?:scan|pq)_\w+)\s*\(',
                                     text)))
    assert declared and sorted(scan.EXPORTED) == declared
    for name in declared:
        assert hasattr(_lib.LIB, name), name


def test_workspace_bytes():
    small = scan.workspace_bytes(8, 4096, 64)
    assert small > 0
    assert scan.workspace_bytes(8, 1 << 20, 64) > small
    big = scan.workspace_bytes(8, 1 << 20, 64)
    assert scan.workspace_bytes(8, 1 << 20, 256) > big  # re-scan lists
    for bad in ((8, 4096, 0), (8, 4096, 257), (-1, 10, 4), (2, -1, 4)):
        assert scan.workspace_bytes(*bad) == 0


def test_wrapper_rejects_host_tensors_and_bad_arguments():
    q = torch.zeros(2, 8)
    r = torch.zeros(10, 8)
    with pytest.raises(ValueError):
        scan.l2_topk(q, r, 4)
    with pytest.raises(ValueError):
        scan.pq_topk(torch.zeros(2, 4, 256), torch.zeros(10, 4,
                                                         dtype=torch.uint8), 4)
    with pytest.raises(ValueError):
        scan.pq_distance_tables(q, torch.zeros(4, 256, 2), 4)


def test_null_and_shape_errors_need_no_gpu():
    a = scan.L2Args()
    assert _lib.LIB.vectra_scan_l2_topk(None, None) == _lib.ERR_NULL
    assert _lib.LIB.vectra_scan_l2_topk(a, None) == _lib.ERR_NULL
    a.queries = a.rows = 0x10000
    a.dimension = 0
    assert _lib.LIB.vectra_scan_l2_topk(a, None) == _lib.ERR_SHAPE
    p = scan.PqArgs()
    p.tables = p.codes = 0x10000
    p.subspaces = 65
    p.code_stride = 65
    assert _lib.LIB.vectra_scan_pq_topk(p, None) == _lib.ERR_SHAPE
    assert _lib.LIB.vectra_pq_distance_tables(
        0x10000, 1, 8, 0x10000, 8, 3, 0x10000, None) == _lib.ERR_SHAPE


def test_level_plan_launch_counts():
    # bench.py's count of a scan call's launches (a level kernel and a
    # select per level, plus the two of the overflow re-scan): one level up
    # to 32,768 candidates, two for the L2 bench (1 M rows, k = 64), three
    # for the PQ bench (16 M codes) and for k = 256 over 1 M rows.
    import bench  # pylint: disable=import-outside-toplevel
    assert bench.scan_launches(1000, 64) == 2
    assert bench.scan_launches(32768, 256) == 2
    assert bench.scan_launches(1 << 20, 64) == 6
    assert bench.scan_launches(1 << 24, 64) == 8
    assert bench.scan_launches(1 << 20, 256) == 8


def test_static_scratch_covers_the_bench_scan():
    # vectra_scan_l2_topk_noalloc serves the L2 bench's shape (8 queries
    # over 1 M rows, k = 64) from its 8 MB static scratch.
    assert 0 < scan.workspace_bytes(8, 1 << 20, 64) <= \
        scan.NOALLOC_SCRATCH_BYTES
