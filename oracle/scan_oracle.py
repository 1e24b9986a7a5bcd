"""Test infrastructure: a CPU restatement of the reference engine's candidate
scoring (the scan path), the checker for vectra_b200.scan.

Only tests/ and bench.py's CPU baseline import this module; the shipped
scan never calls it.

* `l2_squared` restates L2SquaredDistance (engine/src/index/simd_distance.cc:
  36-51) in float32 with its exact order: sixteen lane sums over strided
  elements, a pairwise tree (ReduceLanes, :28-33), then the tail; as written
  (no fused multiply-add), like the reference built by oracle/Makefile.
* `pq_adc` restates PqAdcDistance (:71-85): four chains, (l0 + l1) +
  (l2 + l3), then the tail.
* `distance_tables` restates ProductQuantizer::ComputeDistanceTable
  (engine/src/index/pq_codec.cc:208-217).
* `topk` orders candidates by CloserFirst (engine/include/vectra/index/
  search_scratch.h:35-40: distance, then node id) and keeps k — the result
  of ShardIndex::ExhaustiveSearch's bounded heap and final sort
  (engine/src/index/shard_index.cc:110-120, 236-266).

`load_reference()` loads oracle/_ref/libvectra_engine_ref.so, the reference's
own sources compiled by oracle/Makefile, when it has been built; the CPU
tests pin this restatement to it bit for bit.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

LANES = 16
CENTROIDS = 256
REF_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), '_ref')
REF_LIB = os.path.join(REF_DIR, 'libvectra_engine_ref.so')
# The same sources with the reference's Release flags (the timed baseline).
REF_FAST_LIB = os.path.join(REF_DIR, 'libvectra_engine_ref_fast.so')


def l2_squared(query: np.ndarray, rows: np.ndarray) -> np.ndarray:
    """float32 [N]: L2SquaredDistance(query, row) for each row [N, d]."""
    q = np.asarray(query, np.float32)
    r = np.asarray(rows, np.float32)
    d = q.shape[-1]
    sq = (q[None, :] - r)
    sq = sq * sq  # float32 rounding of each product, as written
    lanes = np.zeros((r.shape[0], LANES), np.float32)
    i = 0
    while i + LANES <= d:
        lanes = lanes + sq[:, i:i + LANES]
        i += LANES
    width = LANES // 2
    while width > 0:
        lanes[:, :width] = lanes[:, :width] + lanes[:, width:2 * width]
        width //= 2
    total = lanes[:, 0].copy()
    for j in range(i, d):
        total = total + sq[:, j]
    return total.astype(np.float32)


def pq_adc(table: np.ndarray, codes: np.ndarray) -> np.ndarray:
    """float32 [N]: PqAdcDistance(table [m, 256], code) for codes [N, m]."""
    t = np.asarray(table, np.float32)
    c = np.asarray(codes, np.uint8)
    m = t.shape[0]
    vals = t[np.arange(m)[None, :], c[:, :m].astype(np.int64)]  # [N, m]
    lanes = [np.zeros(c.shape[0], np.float32) for _ in range(4)]
    s = 0
    while s + 4 <= m:
        for j in range(4):
            lanes[j] = lanes[j] + vals[:, s + j]
        s += 4
    total = (lanes[0] + lanes[1]) + (lanes[2] + lanes[3])
    for j in range(s, m):
        total = total + vals[:, j]
    return total.astype(np.float32)


def distance_tables(queries: np.ndarray, codebooks: np.ndarray) -> np.ndarray:
    """float32 [Q, m, 256] from queries [Q, d] and codebooks [m, 256, d/m]."""
    q = np.asarray(queries, np.float32)
    cb = np.asarray(codebooks, np.float32)
    m, _, dsub = cb.shape
    out = np.empty((q.shape[0], m, CENTROIDS), np.float32)
    for qi in range(q.shape[0]):
        for s in range(m):
            out[qi, s] = l2_squared(q[qi, s * dsub:(s + 1) * dsub], cb[s])
    return out


def topk(distances: np.ndarray, nodes: np.ndarray, k: int):
    """The k first (distance, node) pairs in CloserFirst order."""
    order = np.lexsort((nodes, distances))[:k]
    return distances[order], nodes[order]


def exhaustive_l2_topk(query, rows, k, ids=None):
    """ShardIndex::ExhaustiveSearch of one query: (distances, nodes)."""
    nodes = (np.arange(rows.shape[0], dtype=np.int64) if ids is None
             else np.asarray(ids, np.int64))
    d = l2_squared(query, rows[nodes])
    return topk(d, nodes, k)


def pq_topk(table, codes, k, ids=None):
    """The PQ scan of one query: (distances, nodes)."""
    nodes = (np.arange(codes.shape[0], dtype=np.int64) if ids is None
             else np.asarray(ids, np.int64))
    d = pq_adc(table, codes[nodes])
    return topk(d, nodes, k)


class Reference:
    """ctypes view of oracle/_ref/libvectra_engine_ref.so."""

    def __init__(self, path: str = REF_LIB):
        lib = ctypes.CDLL(path)
        f32p = ctypes.POINTER(ctypes.c_float)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        u32p = ctypes.POINTER(ctypes.c_uint32)
        lib.ref_l2_squared_distance.argtypes = [f32p, f32p, ctypes.c_int]
        lib.ref_l2_squared_distance.restype = ctypes.c_float
        lib.ref_pq_adc_distance.argtypes = [f32p, u8p, ctypes.c_int]
        lib.ref_pq_adc_distance.restype = ctypes.c_float
        lib.ref_l2_distances.argtypes = [f32p, f32p, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_int, f32p]
        lib.ref_exhaustive_topk.argtypes = [
            f32p, f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, u32p,
            ctypes.c_int64, ctypes.c_int, f32p, u32p]
        lib.ref_exhaustive_topk.restype = ctypes.c_int
        lib.ref_pq_topk.argtypes = [f32p, u8p, ctypes.c_int64, ctypes.c_int64,
                                    ctypes.c_int, u32p, ctypes.c_int64,
                                    ctypes.c_int, f32p, u32p]
        lib.ref_pq_topk.restype = ctypes.c_int
        lib.ref_pq_distance_table.argtypes = [ctypes.c_int, ctypes.c_int,
                                              f32p, f32p, f32p]
        lib.ref_pq_distance_table.restype = ctypes.c_int
        lib.ref_pq_encode.argtypes = [ctypes.c_int, ctypes.c_int, f32p, f32p,
                                      ctypes.c_int64, u8p]
        lib.ref_pq_encode.restype = ctypes.c_int
        self.lib = lib

    @staticmethod
    def _p(a, ctype):
        return a.ctypes.data_as(ctypes.POINTER(ctype))

    def l2_distances(self, query, rows):
        q = np.ascontiguousarray(query, np.float32)
        r = np.ascontiguousarray(rows, np.float32)
        out = np.empty(r.shape[0], np.float32)
        self.lib.ref_l2_distances(self._p(q, ctypes.c_float),
                                  self._p(r, ctypes.c_float), r.shape[0],
                                  r.shape[1], r.shape[1],
                                  self._p(out, ctypes.c_float))
        return out

    def exhaustive_topk(self, query, rows, k, ids=None):
        q = np.ascontiguousarray(query, np.float32)
        r = np.ascontiguousarray(rows, np.float32)
        idp, nid = None, 0
        if ids is not None:
            ids = np.ascontiguousarray(ids, np.uint32)
            idp, nid = self._p(ids, ctypes.c_uint32), ids.shape[0]
        od = np.empty(k, np.float32)
        on = np.empty(k, np.uint32)
        n = self.lib.ref_exhaustive_topk(
            self._p(q, ctypes.c_float), self._p(r, ctypes.c_float),
            r.shape[0], r.shape[1], r.shape[1], idp, nid, k,
            self._p(od, ctypes.c_float), self._p(on, ctypes.c_uint32))
        return od[:n], on[:n].astype(np.int64)

    def pq_topk(self, table, codes, k, ids=None):
        t = np.ascontiguousarray(table, np.float32)
        c = np.ascontiguousarray(codes, np.uint8)
        idp, nid = None, 0
        if ids is not None:
            ids = np.ascontiguousarray(ids, np.uint32)
            idp, nid = self._p(ids, ctypes.c_uint32), ids.shape[0]
        od = np.empty(k, np.float32)
        on = np.empty(k, np.uint32)
        n = self.lib.ref_pq_topk(
            self._p(t, ctypes.c_float), self._p(c, ctypes.c_uint8),
            c.shape[0], c.shape[1], t.shape[0], idp, nid, k,
            self._p(od, ctypes.c_float), self._p(on, ctypes.c_uint32))
        return od[:n], on[:n].astype(np.int64)

    def pq_adc(self, table, code):
        t = np.ascontiguousarray(table, np.float32)
        c = np.ascontiguousarray(code, np.uint8)
        return self.lib.ref_pq_adc_distance(self._p(t, ctypes.c_float),
                                            self._p(c, ctypes.c_uint8),
                                            t.shape[0])

    def distance_table(self, query, codebooks):
        cb = np.ascontiguousarray(codebooks, np.float32)
        q = np.ascontiguousarray(query, np.float32)
        m = cb.shape[0]
        out = np.empty((m, CENTROIDS), np.float32)
        status = self.lib.ref_pq_distance_table(
            q.shape[0], m, self._p(cb, ctypes.c_float),
            self._p(q, ctypes.c_float), self._p(out, ctypes.c_float))
        if status != 0:
            raise ValueError('the reference rejected the codebooks')
        return out

    def encode(self, vectors, codebooks):
        cb = np.ascontiguousarray(codebooks, np.float32)
        v = np.ascontiguousarray(vectors, np.float32)
        m = cb.shape[0]
        out = np.empty((v.shape[0], m), np.uint8)
        status = self.lib.ref_pq_encode(v.shape[1], m,
                                        self._p(cb, ctypes.c_float),
                                        self._p(v, ctypes.c_float),
                                        v.shape[0],
                                        self._p(out, ctypes.c_uint8))
        if status != 0:
            raise ValueError('the reference rejected the codebooks')
        return out


def load_reference(fast: bool = False):
    """The compiled reference (the checker build, or with fast=True the
    Release build that bench.py times), or None when oracle/_ref has not
    been built (it needs the reference sources; see oracle/Makefile) or
    cannot load on this host."""
    path = REF_FAST_LIB if fast else REF_LIB
    if not os.path.exists(path):
        return None
    try:
        return Reference(path)
    except OSError:
        return None
