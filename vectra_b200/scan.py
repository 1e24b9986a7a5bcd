"""Exhaustive top-k scans of an index shard on B200 (include/vectra_scan.h).

GPU counterparts of the reference engine's candidate scoring, batched over
queries:

* `l2_topk` replaces ShardIndex::ExhaustiveSearch
  (engine/src/index/shard_index.cc:236-266): the k rows nearest to each
  query by squared L2 distance (L2SquaredDistance,
  engine/src/index/simd_distance.cc:36-51), sorted as CloserFirst sorts them
  (distance, then node id; engine/include/vectra/index/search_scratch.h:
  35-40);
* `pq_topk` does the same over product-quantized codes with PqAdcDistance
  (simd_distance.cc:71-85), given each query's distance table;
* `pq_distance_tables` replaces ProductQuantizer::ComputeDistanceTable
  (engine/src/index/pq_codec.cc:208-217).

Candidates are every row, or per query a list of row ids. Tensors are CUDA
tensors; calls run on the current stream. Results: distances float32
[Q, k], nodes int32 [Q, k] (-1 past a query's count), counts int32 [Q].
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from vectra_b200 import _lib

MAX_K = 256
MAX_SUBSPACES = 64
CENTROIDS = 256

# Every symbol include/vectra_scan.h declares.
EXPORTED = (
    'vectra_scan_workspace_bytes',
    'vectra_scan_l2_topk',
    'vectra_scan_l2_topk_noalloc',
    'vectra_scan_pq_topk',
    'vectra_pq_distance_tables',
)
# Scratch of vectra_scan_l2_topk_noalloc (VECTRA_SCAN_NOALLOC_SCRATCH_BYTES).
NOALLOC_SCRATCH_BYTES = 8 << 20


class Candidates(ctypes.Structure):
    """vectra_scan_candidates."""
    _fields_ = [('offsets', ctypes.c_void_p), ('ids', ctypes.c_void_p),
                ('max_per_query', ctypes.c_int64)]


class Results(ctypes.Structure):
    """vectra_scan_results."""
    _fields_ = [('distances', ctypes.c_void_p), ('nodes', ctypes.c_void_p),
                ('counts', ctypes.c_void_p)]


class L2Args(ctypes.Structure):
    """vectra_scan_l2_args."""
    _fields_ = [('queries', ctypes.c_void_p), ('n_queries', ctypes.c_int64),
                ('query_stride', ctypes.c_int64), ('rows', ctypes.c_void_p),
                ('n_rows', ctypes.c_int64), ('row_stride', ctypes.c_int64),
                ('dimension', ctypes.c_int32), ('k', ctypes.c_int32),
                ('candidates', Candidates), ('results', Results),
                ('workspace', ctypes.c_void_p),
                ('workspace_bytes', ctypes.c_size_t)]


class PqArgs(ctypes.Structure):
    """vectra_scan_pq_args."""
    _fields_ = [('tables', ctypes.c_void_p), ('n_queries', ctypes.c_int64),
                ('codes', ctypes.c_void_p), ('n_rows', ctypes.c_int64),
                ('code_stride', ctypes.c_int64),
                ('subspaces', ctypes.c_int32), ('k', ctypes.c_int32),
                ('candidates', Candidates), ('results', Results),
                ('workspace', ctypes.c_void_p),
                ('workspace_bytes', ctypes.c_size_t)]


def _bind(lib):
    lib.vectra_scan_workspace_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_int32]
    lib.vectra_scan_workspace_bytes.restype = ctypes.c_size_t
    lib.vectra_scan_l2_topk.argtypes = [ctypes.POINTER(L2Args),
                                        ctypes.c_void_p]
    lib.vectra_scan_l2_topk.restype = ctypes.c_int
    lib.vectra_scan_l2_topk_noalloc.argtypes = [ctypes.POINTER(L2Args),
                                                ctypes.c_void_p]
    lib.vectra_scan_l2_topk_noalloc.restype = ctypes.c_int
    lib.vectra_scan_pq_topk.argtypes = [ctypes.POINTER(PqArgs),
                                        ctypes.c_void_p]
    lib.vectra_scan_pq_topk.restype = ctypes.c_int
    lib.vectra_pq_distance_tables.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
    lib.vectra_pq_distance_tables.restype = ctypes.c_int


_bind(_lib.LIB)


class ScanError(RuntimeError):
    """A scan call returned an error status."""


def _check(status: int, what: str):
    if status != _lib.OK:
        raise ScanError(f'{what}: {_lib.strerror(status)}')


def workspace_bytes(n_queries: int, max_candidates: int, k: int) -> int:
    """Workspace a scan of `n_queries` queries with at most `max_candidates`
    candidates each needs (0 for invalid arguments)."""
    return int(_lib.LIB.vectra_scan_workspace_bytes(n_queries, max_candidates,
                                                    k))


def _cuda(t: torch.Tensor, name: str, dtype) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f'{name} must be a CUDA tensor')
    if t.dtype != dtype:
        raise ValueError(f'{name} must be {dtype}, got {t.dtype}')
    return t


def _candidates(cands, n_queries, device):
    """(Candidates, keep-alive tensors, max per query) from None, a list of
    per-query id tensors, or an (offsets, ids) pair of CUDA tensors."""
    if cands is None:
        return Candidates(None, None, 0), (), None
    if isinstance(cands, tuple):
        offsets, ids = cands
        offsets = _cuda(offsets, 'offsets', torch.int64)
        ids = _cuda(ids, 'ids', torch.int32)
        if offsets.numel() != n_queries + 1:
            raise ValueError('offsets must have n_queries + 1 entries')
        counts = offsets[1:] - offsets[:-1]
        mx = int(counts.max()) if n_queries else 0
    else:
        lists = list(cands)
        if len(lists) != n_queries:
            raise ValueError('one candidate list per query')
        counts = torch.tensor([len(x) for x in lists], dtype=torch.int64)
        offsets = torch.zeros(n_queries + 1, dtype=torch.int64)
        offsets[1:] = torch.cumsum(counts, 0)
        ids = (torch.cat([torch.as_tensor(x, dtype=torch.int64).reshape(-1)
                          for x in lists]) if lists else
               torch.zeros(0, dtype=torch.int64))
        offsets = offsets.to(device)
        ids = ids.to(torch.int32).to(device)
        mx = int(counts.max()) if n_queries else 0
    return (Candidates(offsets.data_ptr(), ids.data_ptr(), mx),
            (offsets, ids), mx)


def _results(n_queries, k, device):
    d = torch.empty(n_queries, k, dtype=torch.float32, device=device)
    n = torch.empty(n_queries, k, dtype=torch.int32, device=device)
    c = torch.empty(n_queries, dtype=torch.int32, device=device)
    return d, n, c, Results(d.data_ptr(), n.data_ptr(), c.data_ptr())


def _workspace(nbytes, device, workspace):
    if workspace is None:
        return torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device)
    if workspace.numel() * workspace.element_size() < nbytes:
        raise ValueError(f'workspace of {nbytes} bytes needed')
    return workspace


def l2_topk_noalloc(queries: torch.Tensor, rows: torch.Tensor, k: int,
                    candidates=None):
    """l2_topk through vectra_scan_l2_topk_noalloc: no workspace (the
    library's static scratch; calls on one device take turns with it)."""
    return l2_topk(queries, rows, k, candidates, _noalloc=True)


def l2_topk(queries: torch.Tensor, rows: torch.Tensor, k: int,
            candidates=None, workspace: torch.Tensor | None = None,
            _noalloc: bool = False):
    """The k rows nearest to each query (squared L2), sorted by (distance,
    node): (distances [Q, k] float32, nodes [Q, k] int32, counts [Q]).

    queries [Q, d] and rows [N, d] are float32 CUDA tensors with unit inner
    stride; candidates: None (every row), a list of Q id sequences, or an
    (offsets int64 [Q + 1], ids int32) pair of CUDA tensors.
    """
    _cuda(queries, 'queries', torch.float32)
    _cuda(rows, 'rows', torch.float32)
    if queries.dim() != 2 or rows.dim() != 2 or \
            queries.shape[1] != rows.shape[1]:
        raise ValueError('queries [Q, d] and rows [N, d] must share d')
    if queries.stride(1) != 1 or rows.stride(1) != 1:
        raise ValueError('queries and rows need unit inner stride')
    if not 1 <= k <= MAX_K:
        raise ValueError(f'k must be in 1..{MAX_K}')
    nq, d = queries.shape
    cand, keep, mx = _candidates(candidates, nq, queries.device)
    dist, nodes, counts, res = _results(nq, k, queries.device)
    stream = torch.cuda.current_stream(queries.device).cuda_stream
    if _noalloc:
        a = L2Args(queries.data_ptr(), nq, queries.stride(0), rows.data_ptr(),
                   rows.shape[0], rows.stride(0), d, k, cand, res, None, 0)
        _check(_lib.LIB.vectra_scan_l2_topk_noalloc(
            ctypes.byref(a), ctypes.c_void_p(stream)),
               'vectra_scan_l2_topk_noalloc')
        del keep
        return dist, nodes, counts
    need = workspace_bytes(nq, rows.shape[0] if mx is None else mx, k)
    ws = _workspace(need, queries.device, workspace)
    a = L2Args(queries.data_ptr(), nq, queries.stride(0), rows.data_ptr(),
               rows.shape[0], rows.stride(0), d, k, cand, res, ws.data_ptr(),
               ws.numel() * ws.element_size())
    _check(_lib.LIB.vectra_scan_l2_topk(ctypes.byref(a),
                                        ctypes.c_void_p(stream)),
           'vectra_scan_l2_topk')
    del keep
    return dist, nodes, counts


def pq_topk(tables: torch.Tensor, codes: torch.Tensor, k: int,
            candidates=None, workspace: torch.Tensor | None = None):
    """The k rows nearest to each query by PQ asymmetric distance: tables
    [Q, m, 256] float32, codes [N, m'] uint8 (m' >= m, unit inner stride).
    Returns (distances, nodes, counts) as l2_topk does."""
    _cuda(tables, 'tables', torch.float32)
    _cuda(codes, 'codes', torch.uint8)
    if tables.dim() != 3 or tables.shape[2] != CENTROIDS or \
            not tables.is_contiguous():
        raise ValueError('tables must be contiguous [Q, m, 256]')
    if codes.dim() != 2 or codes.stride(1) != 1 or \
            codes.shape[1] < tables.shape[1]:
        raise ValueError('codes must be [N, >= m] with unit inner stride')
    nq, m, _ = tables.shape
    if not 1 <= m <= MAX_SUBSPACES:
        raise ValueError(f'm must be in 1..{MAX_SUBSPACES}')
    if not 1 <= k <= MAX_K:
        raise ValueError(f'k must be in 1..{MAX_K}')
    cand, keep, mx = _candidates(candidates, nq, tables.device)
    dist, nodes, counts, res = _results(nq, k, tables.device)
    need = workspace_bytes(nq, codes.shape[0] if mx is None else mx, k)
    ws = _workspace(need, tables.device, workspace)
    a = PqArgs(tables.data_ptr(), nq, codes.data_ptr(), codes.shape[0],
               codes.stride(0), m, k, cand, res, ws.data_ptr(),
               ws.numel() * ws.element_size())
    stream = torch.cuda.current_stream(tables.device).cuda_stream
    _check(_lib.LIB.vectra_scan_pq_topk(ctypes.byref(a),
                                        ctypes.c_void_p(stream)),
           'vectra_scan_pq_topk')
    del keep
    return dist, nodes, counts


def pq_distance_tables(queries: torch.Tensor, codebooks: torch.Tensor,
                       subspaces: int) -> torch.Tensor:
    """[Q, m, 256] squared distances from each query sub-vector to each
    centroid of its sub-space; codebooks [m, 256, d / m] float32 (the
    reference's [subspace][centroid][sub-dimension] layout)."""
    _cuda(queries, 'queries', torch.float32)
    _cuda(codebooks, 'codebooks', torch.float32)
    nq, d = queries.shape
    if d % subspaces or codebooks.shape != (subspaces, CENTROIDS,
                                            d // subspaces) or \
            not codebooks.is_contiguous() or queries.stride(1) != 1:
        raise ValueError('codebooks must be contiguous [m, 256, d / m]')
    out = torch.empty(nq, subspaces, CENTROIDS, dtype=torch.float32,
                      device=queries.device)
    stream = torch.cuda.current_stream(queries.device).cuda_stream
    _check(_lib.LIB.vectra_pq_distance_tables(
        queries.data_ptr(), nq, queries.stride(0), codebooks.data_ptr(), d,
        subspaces, out.data_ptr(), ctypes.c_void_p(stream)),
           'vectra_pq_distance_tables')
    return out


def stack_lists(lists: Sequence[Sequence[int]], device):
    """(offsets, ids) CUDA tensors of per-query candidate id lists."""
    _, keep, _ = _candidates(lists, len(lists), device)
    return keep
