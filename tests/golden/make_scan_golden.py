"""Generates tests/golden/scan_golden.npz: seeded inputs of the scan path
and the outputs of the reference engine's own code for them.

The outputs come from oracle/_ref/libvectra_engine_ref.so, the reference's
simd_distance.cc and pq_codec.cc compiled where they lie (oracle/Makefile),
through its C shim: ExhaustiveSearch's bounded top-k over
L2SquaredDistance, the same over PqAdcDistance, ComputeDistanceTable and
Encode. Run in a checkout that has the reference:

    make -C oracle && python tests/golden/make_scan_golden.py
"""

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(
    os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import scan_oracle  # noqa: E402  pylint: disable=wrong-import-position

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)),
                   'scan_golden.npz')

# (name, dimension, rows, k, with per-query candidate ids)
L2_CASES = [('l2_d1', 1, 300, 5, False), ('l2_d17', 17, 400, 10, False),
            ('l2_d64', 64, 500, 64, False), ('l2_d100', 100, 300, 33, True),
            ('l2_d128_k1', 128, 256, 1, True)]
# (name, sub-spaces, rows, k)
PQ_CASES = [('pq_m1', 1, 300, 7), ('pq_m3', 3, 300, 20), ('pq_m8', 8, 500, 64),
            ('pq_m16', 16, 600, 50), ('pq_m17', 17, 300, 9)]


def main():
    ref = scan_oracle.load_reference()
    if ref is None:
        raise SystemExit('build oracle/_ref first: make -C oracle')
    rng = np.random.default_rng(2024)
    out = {}
    for name, d, n, k, with_ids in L2_CASES:
        rows = rng.standard_normal((n, d)).astype(np.float32)
        queries = (rows[rng.integers(0, n, 3)] +
                   0.1 * rng.standard_normal((3, d))).astype(np.float32)
        out[f'{name}/rows'] = rows
        out[f'{name}/queries'] = queries
        for qi in range(3):
            ids = None
            if with_ids:
                ids = np.sort(rng.choice(n, size=n // 3, replace=False)
                              ).astype(np.uint32)
                out[f'{name}/ids{qi}'] = ids
            dist, nodes = ref.exhaustive_topk(queries[qi], rows, k, ids)
            out[f'{name}/dist{qi}'] = dist
            out[f'{name}/nodes{qi}'] = nodes
    for name, m, n, k in PQ_CASES:
        dsub = 4
        codebooks = rng.standard_normal((m, 256, dsub)).astype(np.float32)
        vectors = rng.standard_normal((n, m * dsub)).astype(np.float32)
        codes = ref.encode(vectors, codebooks)
        query = rng.standard_normal(m * dsub).astype(np.float32)
        table = ref.distance_table(query, codebooks)
        dist, nodes = ref.pq_topk(table, codes, k)
        out[f'{name}/codebooks'] = codebooks
        out[f'{name}/codes'] = codes
        out[f'{name}/query'] = query
        out[f'{name}/table'] = table
        out[f'{name}/dist'] = dist
        out[f'{name}/nodes'] = nodes
    np.savez_compressed(OUT, **out)
    print(f'wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(out)} arrays)')


if __name__ == '__main__':
    main()
