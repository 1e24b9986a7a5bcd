/* vectra_scan.h — exhaustive top-k scans of an index shard on B200 (sm_100a).
 *
 * GPU counterparts of the reference engine's candidate scoring, for a batch
 * of queries per call:
 *  - vectra_scan_l2_topk replaces ShardIndex::ExhaustiveSearch
 *    (engine/src/index/shard_index.cc:236-266): the squared L2 distance
 *    (L2SquaredDistance, engine/src/index/simd_distance.cc:36-51) from the
 *    query to every candidate row, the k nearest kept in the order of
 *    CloserFirst (engine/include/vectra/index/search_scratch.h:35-40:
 *    distance, then node id), returned sorted;
 *  - vectra_scan_pq_topk does the same with PqAdcDistance
 *    (simd_distance.cc:71-85) over product-quantized codes, given each
 *    query's distance table;
 *  - vectra_pq_distance_tables replaces ProductQuantizer::
 *    ComputeDistanceTable (engine/src/index/pq_codec.cc:208-217).
 * Candidates are every row, or per query a list of row ids (the geofilter's
 * cell ranges of shard_index.cc:254-260 flattened to ids).
 *
 * Every call is asynchronous on the given CUDA stream; pointers are device
 * pointers; the caller owns every buffer, including a workspace sized by
 * vectra_scan_workspace_bytes. Status codes are those of vectra_rbf.h. The
 * kernels' waits on their own copies are bounded: one that runs out sets a
 * bit of the device error word that vectra_rbf_check_device_errors reports,
 * and the kernel returns.
 */
#ifndef VECTRA_SCAN_H_
#define VECTRA_SCAN_H_

#include <stddef.h>
#include <stdint.h>

#include "vectra_rbf.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Largest k of one scan (the reference's rerank_depth defaults to 64,
 * engine/include/vectra/index/shard_index.h:48). */
#define VECTRA_SCAN_MAX_K 256
/* Largest number of PQ sub-spaces (code bytes per row). */
#define VECTRA_SCAN_MAX_SUBSPACES 64
/* Centroids per PQ sub-space (kPqCentroids, simd_distance.h). */
#define VECTRA_PQ_CENTROIDS 256

/* Candidates of each query: NULL offsets = every row 0..n_rows-1; else query
 * q scans ids[offsets[q] .. offsets[q + 1]) (row ids < n_rows), and
 * max_per_query bounds offsets[q + 1] - offsets[q] (it sizes the grid, so
 * the call needs no read-back of the offsets). */
typedef struct {
  const int64_t* offsets; /* [n_queries + 1], offsets[0] == 0 */
  const uint32_t* ids;
  int64_t max_per_query;
} vectra_scan_candidates;

/* Results: the k nearest candidates of each query, ascending by (distance,
 * node); a query with fewer than k candidates has (+inf, UINT32_MAX) in the
 * slots past its count. */
typedef struct {
  float* distances;  /* [n_queries][k] */
  uint32_t* nodes;   /* [n_queries][k] */
  int32_t* counts;   /* [n_queries] min(k, candidates); may be NULL */
} vectra_scan_results;

typedef struct {
  const float* queries;   /* [n_queries][query_stride] */
  int64_t n_queries;
  int64_t query_stride;   /* floats, >= dimension */
  const float* rows;      /* [n_rows][row_stride] */
  int64_t n_rows;
  int64_t row_stride;     /* floats, >= dimension */
  int32_t dimension;      /* 1..4096 */
  int32_t k;              /* 1..VECTRA_SCAN_MAX_K */
  vectra_scan_candidates candidates;
  vectra_scan_results results;
  void* workspace;        /* 16-byte aligned */
  size_t workspace_bytes;
} vectra_scan_l2_args;

typedef struct {
  const float* tables;    /* [n_queries][subspaces][VECTRA_PQ_CENTROIDS] */
  int64_t n_queries;
  const uint8_t* codes;   /* [n_rows][code_stride] */
  int64_t n_rows;
  int64_t code_stride;    /* bytes, >= subspaces */
  int32_t subspaces;      /* 1..VECTRA_SCAN_MAX_SUBSPACES */
  int32_t k;              /* 1..VECTRA_SCAN_MAX_K */
  vectra_scan_candidates candidates;
  vectra_scan_results results;
  void* workspace;        /* 16-byte aligned */
  size_t workspace_bytes;
} vectra_scan_pq_args;

/* Workspace bytes for a scan of n_queries queries with at most
 * max_candidates candidates each (n_rows for a scan of every row). */
VECTRA_API size_t vectra_scan_workspace_bytes(int64_t n_queries,
                                              int64_t max_candidates,
                                              int32_t k);

/* Replaces ShardIndex::ExhaustiveSearch (shard_index.cc:236-266). */
VECTRA_API int vectra_scan_l2_topk(const vectra_scan_l2_args* args,
                                   void* stream);

/* The PQ scan: distance of a row = sum over sub-spaces s of
 * tables[q][s][codes[row][s]] (PqAdcDistance, simd_distance.cc:71-85,
 * summed in its order). */
VECTRA_API int vectra_scan_pq_topk(const vectra_scan_pq_args* args,
                                   void* stream);

/* vectra_scan_l2_topk for callers that cannot allocate device memory: a
 * host bound through an FFI (cgo, JNI, ctypes) that is handed device
 * pointers but has no CUDA allocator of its own, or a serving loop that
 * allows no cudaMalloc after start-up (it synchronizes the device and can
 * fail under memory pressure). The caller passes inputs and outputs only;
 * the scan's scratch is a static array of VECTRA_SCAN_NOALLOC_SCRATCH_BYTES
 * (8 MB) built into the library, which every GPU that loads the library
 * holds until the process exits. args->workspace is ignored.
 * VECTRA_ERR_UNSUPPORTED when the scan needs more scratch than that
 * (vectra_scan_workspace_bytes above VECTRA_SCAN_NOALLOC_SCRATCH_BYTES).
 * The first call on a device, with that device current, does the set-up:
 * it looks up the array's device address and creates one event, so that
 * first call should come before any stream capture. Both stay cached for
 * the life of the process, so after a cudaDeviceReset of a device this
 * entry point must not be called on that device again. Every call on a
 * device shares the array, and two calls in flight on the GPU at once
 * would race on it, so each call's stream first waits for the previous
 * call's kernels, whatever stream they ran on. A
 * call writes every part of the array that it reads; nothing carries over
 * from the last call.
 * No counterpart in the reference: an entry point of this library only. */
#define VECTRA_SCAN_NOALLOC_SCRATCH_BYTES (8u << 20)
VECTRA_API int vectra_scan_l2_topk_noalloc(const vectra_scan_l2_args* args,
                                           void* stream);

/* tables[q][s][c] = squared L2 distance from sub-vector s of query q to
 * centroid c of sub-space s; codebooks laid out [subspace][centroid]
 * [dimension / subspaces] as ProductQuantizer stores them
 * (pq_codec.h: FromCodebooks). Replaces ComputeDistanceTable
 * (pq_codec.cc:208-217). */
VECTRA_API int vectra_pq_distance_tables(const float* queries,
                                         int64_t n_queries,
                                         int64_t query_stride,
                                         const float* codebooks,
                                         int32_t dimension, int32_t subspaces,
                                         float* tables, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VECTRA_SCAN_H_ */
