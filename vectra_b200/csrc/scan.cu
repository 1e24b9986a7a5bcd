// scan.cu: exhaustive top-k scans of an index shard (include/vectra_scan.h),
// the GPU counterparts of the reference engine's candidate scoring:
// ShardIndex::ExhaustiveSearch (engine/src/index/shard_index.cc:236-266),
// L2SquaredDistance / PqAdcDistance (engine/src/index/simd_distance.cc) and
// ProductQuantizer::ComputeDistanceTable (engine/src/index/pq_codec.cc).
//
// Design (B200):
//  * Candidates are scanned in tiles of kTile = 4,096; a CTA of 8 warps
//    takes one tile for a group of QG queries (the queries' vectors, or
//    their PQ tables, in shared memory). Blocks are ordered tile-major, so
//    the CTAs of all query groups of a tile run together and read the tile
//    from HBM once (L2 serves the others).
//  * Lane per candidate row: the lane reads its row with 16-byte loads
//    (read-only path) and forms the distance to each of the QG queries:
//    sum_d (q_d - r_d)^2 in float32 with packed f32x2 subtract/FMA (the
//    reference formulation, direct differences); for PQ the sum of the
//    table entries of its code bytes, in PqAdcDistance's order (four chains,
//    (l0 + l1) + (l2 + l3), then the tail: bit-identical sums).
//  * Top-k: each warp keeps, per query, a sorted list of k (distance, node)
//    pairs spread over its lanes' registers (entry j at lane j % 32, slot
//    j / 32), ordered as CloserFirst orders them (distance, then node id;
//    engine/include/vectra/index/search_scratch.h:35-40). Each batch of 32
//    candidates is filtered by the list's last entry (a ballot); survivors
//    are inserted one at a time by a warp-wide shift (shuffles). After the
//    tile, the CTA's warps merge their lists (warp g merges query g) and
//    write the tile's top k to the workspace; a second kernel merges a
//    query's tiles the same way and writes the sorted result.
#include <math.h>
#include <stdint.h>

#include <atomic>

#include "rbf_common.cuh"
#include "vectra_scan.h"

namespace vectra {
namespace scan {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerLane = 16;
constexpr int kTile = kThreads * kRowsPerLane;  // candidates per CTA tile
constexpr uint32_t kNoNode = 0xffffffffu;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ bool closer(float da, uint32_t na, float db,
                                       uint32_t nb) {
  return da < db || (da == db && na < nb);
}

// A sorted list of K <= 32 * KPW pairs spread over the warp: entry j at lane
// j % 32, slot j / 32. Entries past the filled part are (+inf, kNoNode).
template <int KPW>
struct WarpList {
  float d[KPW];
  uint32_t n[KPW];

  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int s = 0; s < KPW; ++s) {
      d[s] = INFINITY;
      n[s] = kNoNode;
    }
  }
  // The last entry of a list of k (the admission threshold), on every lane.
  __device__ __forceinline__ void last(int k, float& td, uint32_t& tn) const {
    const int s = (k - 1) >> 5, l = (k - 1) & 31;
    float dv = d[0];
    uint32_t nv = n[0];
#pragma unroll
    for (int i = 1; i < KPW; ++i)
      if (i == s) {
        dv = d[i];
        nv = n[i];
      }
    td = __shfl_sync(kFull, dv, l);
    tn = __shfl_sync(kFull, nv, l);
  }
  // Inserts (cd, cn), which is closer than the current last entry: entries
  // from its position on move up by one and the last one drops off.
  __device__ __forceinline__ void insert(float cd, uint32_t cn, int k,
                                         int lane) {
    int pos = 0;
#pragma unroll
    for (int s = 0; s < KPW; ++s)
      pos += __popc(__ballot_sync(kFull, closer(d[s], n[s], cd, cn)));
    float nd[KPW];
    uint32_t nn[KPW];
#pragma unroll
    for (int s = 0; s < KPW; ++s) {
      float ud = __shfl_up_sync(kFull, d[s], 1);
      uint32_t un = __shfl_up_sync(kFull, n[s], 1);
      if (s > 0) {
        const float cd0 = __shfl_sync(kFull, d[s - 1], 31);
        const uint32_t cn0 = __shfl_sync(kFull, n[s - 1], 31);
        if (lane == 0) {
          ud = cd0;
          un = cn0;
        }
      }
      const int j = s * 32 + lane;
      if (j >= k) {
        nd[s] = INFINITY;
        nn[s] = kNoNode;
      } else if (j > pos) {
        nd[s] = ud;
        nn[s] = un;
      } else if (j == pos) {
        nd[s] = cd;
        nn[s] = cn;
      } else {
        nd[s] = d[s];
        nn[s] = n[s];
      }
    }
#pragma unroll
    for (int s = 0; s < KPW; ++s) {
      d[s] = nd[s];
      n[s] = nn[s];
    }
  }
  // Offers one candidate per lane (+inf for none).
  __device__ __forceinline__ void offer(float cd, uint32_t cn, int k,
                                        int lane) {
    float td;
    uint32_t tn;
    last(k, td, tn);
    unsigned pass = __ballot_sync(kFull, closer(cd, cn, td, tn));
    while (pass) {
      const int b = __ffs(pass) - 1;
      pass &= pass - 1;
      const float bd = __shfl_sync(kFull, cd, b);
      const uint32_t bn = __shfl_sync(kFull, cn, b);
      if (closer(bd, bn, td, tn)) {  // the threshold may have moved
        insert(bd, bn, k, lane);
        last(k, td, tn);
      }
    }
  }
};

// Packed float pairs (sm_100a f32x2 arithmetic).
__device__ __forceinline__ uint64_t pk(float x, float y) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
  return r;
}
__device__ __forceinline__ float2 upk(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

struct ScanShape {
  int64_t n_queries;
  int64_t n_rows;
  int64_t n_tiles;        // tiles per query (of the largest candidate set)
  const int64_t* offsets;  // per-query candidates (CSR), or null
  const uint32_t* ids;
  int k;
};

// Candidate i of query q's tile-relative range: its node id, or kNoNode.
__device__ __forceinline__ uint32_t candidate(const ScanShape& sh, int64_t q,
                                              int64_t i) {
  if (sh.offsets == nullptr) return i < sh.n_rows ? uint32_t(i) : kNoNode;
  const int64_t lo = sh.offsets[q], hi = sh.offsets[q + 1];
  return lo + i < hi ? sh.ids[lo + i] : kNoNode;
}

// The CTA's per-warp lists of query g are written to smem; warp g merges
// them and writes the tile's top k to the workspace.
template <int KPW, int QG>
__device__ __forceinline__ void merge_tile(WarpList<KPW> (&lists)[QG],
                                           float* sd, uint32_t* sn,
                                           int64_t q0, int64_t nq, int64_t tile,
                                           const ScanShape& sh, float* wd,
                                           uint32_t* wn) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k = sh.k;
  constexpr int KP = KPW * 32;  // padded list length
#pragma unroll
  for (int g = 0; g < QG; ++g)
#pragma unroll
    for (int s = 0; s < KPW; ++s) {
      const int idx = (g * kWarps + warp) * KP + s * 32 + lane;
      sd[idx] = lists[g].d[s];
      sn[idx] = lists[g].n[s];
    }
  __syncthreads();
  for (int g = warp; g < QG; g += kWarps) {
    if (q0 + g >= nq) continue;
    WarpList<KPW> m;
#pragma unroll
    for (int s = 0; s < KPW; ++s) {
      m.d[s] = sd[(g * kWarps) * KP + s * 32 + lane];
      m.n[s] = sn[(g * kWarps) * KP + s * 32 + lane];
    }
    for (int i = KP; i < kWarps * KP; i += 32) {
      const int idx = g * kWarps * KP + i + lane;
      m.offer(sd[idx], sn[idx], k, lane);
    }
    const size_t base = (size_t(q0 + g) * sh.n_tiles + tile) * KP;
#pragma unroll
    for (int s = 0; s < KPW; ++s) {
      wd[base + s * 32 + lane] = m.d[s];
      wn[base + s * 32 + lane] = m.n[s];
    }
  }
}

// ---------------------------------------------------------------------------
// L2 scan.
// ---------------------------------------------------------------------------
template <int KPW, int QG>
__global__ void __launch_bounds__(kThreads)
    l2_scan_kernel(const float* __restrict__ queries, int64_t query_stride,
                   const float* __restrict__ rows, int64_t row_stride,
                   int dim, int vec4, ScanShape sh, float* wd, uint32_t* wn) {
  extern __shared__ __align__(16) float smem_f[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_groups = (sh.n_queries + QG - 1) / QG;
  const int64_t group = blockIdx.x % n_groups;
  const int64_t tile = blockIdx.x / n_groups;
  const int64_t q0 = group * QG;
  const int dpad = (dim + 3) & ~3;
  float* sq = smem_f;                         // [QG][dpad]
  float* sd = sq + QG * dpad;                 // merge area
  uint32_t* sn = reinterpret_cast<uint32_t*>(sd + QG * kWarps * KPW * 32);
  for (int i = threadIdx.x; i < QG * dpad; i += kThreads) {
    const int g = i / dpad, c = i - g * dpad;
    sq[i] = (q0 + g < sh.n_queries && c < dim)
                ? queries[(q0 + g) * query_stride + c]
                : 0.f;
  }
  __syncthreads();

  WarpList<KPW> lists[QG];
#pragma unroll
  for (int g = 0; g < QG; ++g) lists[g].clear();
  for (int r = 0; r < kRowsPerLane; ++r) {
    const int64_t i = tile * kTile + (int64_t(r) * kWarps + warp) * 32 + lane;
    // Candidates of a group's queries coincide (per-query lists use QG = 1).
    const uint32_t node = candidate(sh, q0, i);
    float dist[QG];
    if (node != kNoNode) {
      const float* row = rows + int64_t(node) * row_stride;
      uint64_t acc[QG][2];
#pragma unroll
      for (int g = 0; g < QG; ++g) acc[g][0] = acc[g][1] = 0;
      if (vec4) {
        for (int c = 0; c < dim; c += 4) {
          const float4 rv = __ldg(reinterpret_cast<const float4*>(row + c));
          const uint64_t r01 = pk(rv.x, rv.y), r23 = pk(rv.z, rv.w);
#pragma unroll
          for (int g = 0; g < QG; ++g) {
            const float4 qv = *reinterpret_cast<const float4*>(sq + g * dpad + c);
            const uint64_t d01 = sub2(pk(qv.x, qv.y), r01);
            const uint64_t d23 = sub2(pk(qv.z, qv.w), r23);
            acc[g][0] = fma2(d01, d01, acc[g][0]);
            acc[g][1] = fma2(d23, d23, acc[g][1]);
          }
        }
      } else {
        for (int c = 0; c < dim; ++c) {
          const float rv = __ldg(row + c);
#pragma unroll
          for (int g = 0; g < QG; ++g) {
            const uint64_t dd = pk(sq[g * dpad + c] - rv, 0.f);
            acc[g][c & 1] = fma2(dd, dd, acc[g][c & 1]);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < QG; ++g) {
        const float2 a = upk(acc[g][0]), b = upk(acc[g][1]);
        dist[g] = (a.x + a.y) + (b.x + b.y);
      }
    } else {
#pragma unroll
      for (int g = 0; g < QG; ++g) dist[g] = INFINITY;
    }
#pragma unroll
    for (int g = 0; g < QG; ++g) lists[g].offer(dist[g], node, sh.k, lane);
  }
  merge_tile<KPW, QG>(lists, sd, sn, q0, sh.n_queries, tile, sh, wd, wn);
}

// ---------------------------------------------------------------------------
// PQ (asymmetric distance) scan.
// ---------------------------------------------------------------------------
template <int KPW, int QG>
__global__ void __launch_bounds__(kThreads)
    pq_scan_kernel(const float* __restrict__ tables,
                   const uint8_t* __restrict__ codes, int64_t code_stride,
                   int m, int vec16, ScanShape sh, float* wd, uint32_t* wn) {
  extern __shared__ __align__(16) float smem_f[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_groups = (sh.n_queries + QG - 1) / QG;
  const int64_t group = blockIdx.x % n_groups;
  const int64_t tile = blockIdx.x / n_groups;
  const int64_t q0 = group * QG;
  const int tsz = m * VECTRA_PQ_CENTROIDS;
  float* st = smem_f;                          // [QG][m][256]
  float* sd = st + QG * tsz;
  uint32_t* sn = reinterpret_cast<uint32_t*>(sd + QG * kWarps * KPW * 32);
  for (int i = threadIdx.x; i < QG * tsz; i += kThreads) {
    const int g = i / tsz;
    st[i] = q0 + g < sh.n_queries ? tables[(q0 + g) * tsz + (i - g * tsz)]
                                  : 0.f;
  }
  __syncthreads();

  WarpList<KPW> lists[QG];
#pragma unroll
  for (int g = 0; g < QG; ++g) lists[g].clear();
  uint8_t code[VECTRA_SCAN_MAX_SUBSPACES];
  for (int r = 0; r < kRowsPerLane; ++r) {
    const int64_t i = tile * kTile + (int64_t(r) * kWarps + warp) * 32 + lane;
    const uint32_t node = candidate(sh, q0, i);
    float dist[QG];
    if (node != kNoNode) {
      const uint8_t* cp = codes + int64_t(node) * code_stride;
      if (vec16) {
        for (int s = 0; s < m; s += 16) {
          const uint4 w = __ldg(reinterpret_cast<const uint4*>(cp + s));
          *reinterpret_cast<uint4*>(code + s) = w;
        }
      } else {
        for (int s = 0; s < m; ++s) code[s] = __ldg(cp + s);
      }
#pragma unroll
      for (int g = 0; g < QG; ++g) {
        // PqAdcDistance (simd_distance.cc:71-85): four chains, then the
        // tail, in this order.
        const float* t = st + g * tsz;
        float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
        int s = 0;
        for (; s + 4 <= m; s += 4) {
          l0 = __fadd_rn(l0, t[(s + 0) * 256 + code[s + 0]]);
          l1 = __fadd_rn(l1, t[(s + 1) * 256 + code[s + 1]]);
          l2 = __fadd_rn(l2, t[(s + 2) * 256 + code[s + 2]]);
          l3 = __fadd_rn(l3, t[(s + 3) * 256 + code[s + 3]]);
        }
        float sum = __fadd_rn(__fadd_rn(l0, l1), __fadd_rn(l2, l3));
        for (; s < m; ++s) sum = __fadd_rn(sum, t[s * 256 + code[s]]);
        dist[g] = sum;
      }
    } else {
#pragma unroll
      for (int g = 0; g < QG; ++g) dist[g] = INFINITY;
    }
#pragma unroll
    for (int g = 0; g < QG; ++g) lists[g].offer(dist[g], node, sh.k, lane);
  }
  merge_tile<KPW, QG>(lists, sd, sn, q0, sh.n_queries, tile, sh, wd, wn);
}

// ---------------------------------------------------------------------------
// Merge of a query's tiles: one warp per query.
// ---------------------------------------------------------------------------
template <int KPW>
__global__ void __launch_bounds__(128)
    merge_kernel(const float* wd, const uint32_t* wn, ScanShape sh,
                 float* out_d, uint32_t* out_n, int32_t* counts) {
  const int lane = threadIdx.x & 31;
  const int64_t q = int64_t(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (q >= sh.n_queries) return;
  constexpr int KP = KPW * 32;
  const int k = sh.k;
  const size_t base = size_t(q) * sh.n_tiles * KP;
  WarpList<KPW> m;
#pragma unroll
  for (int s = 0; s < KPW; ++s) {
    m.d[s] = wd[base + s * 32 + lane];
    m.n[s] = wn[base + s * 32 + lane];
  }
  const int64_t total = sh.n_tiles * KP;
  for (int64_t i = KP; i < total; i += 32)
    m.offer(wd[base + i + lane], wn[base + i + lane], k, lane);
#pragma unroll
  for (int s = 0; s < KPW; ++s) {
    const int j = s * 32 + lane;
    if (j < k) {
      out_d[q * k + j] = m.d[s];
      out_n[q * k + j] = m.n[s];
    }
  }
  if (counts != nullptr) {
    int64_t nc = sh.offsets == nullptr ? sh.n_rows
                                       : sh.offsets[q + 1] - sh.offsets[q];
    if (lane == 0) counts[q] = int32_t(nc < k ? nc : k);
  }
}

// ---------------------------------------------------------------------------
// PQ distance tables.
// ---------------------------------------------------------------------------
// tables[q][s][c] = L2SquaredDistance(query sub-vector s, centroid c of
// sub-space s), in the reference's order (simd_distance.cc:36-51): sixteen
// strided lane sums, a pairwise tree over them, then the tail.
__global__ void __launch_bounds__(256)
    pq_tables_kernel(const float* __restrict__ queries, int64_t n_queries,
                     int64_t query_stride, const float* __restrict__ codebooks,
                     int dsub, int m, float* tables) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = n_queries * m * VECTRA_PQ_CENTROIDS;
  if (idx >= total) return;
  const int c = int(idx % VECTRA_PQ_CENTROIDS);
  const int s = int((idx / VECTRA_PQ_CENTROIDS) % m);
  const int64_t q = idx / (int64_t(m) * VECTRA_PQ_CENTROIDS);
  const float* a = queries + q * query_stride + int64_t(s) * dsub;
  const float* b = codebooks + (int64_t(s) * VECTRA_PQ_CENTROIDS + c) * dsub;
  float lanes[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) lanes[j] = 0.f;
  int i = 0;
  for (; i + 16 <= dsub; i += 16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float d = __fsub_rn(__ldg(a + i + j), __ldg(b + i + j));
      lanes[j] = __fadd_rn(lanes[j], __fmul_rn(d, d));
    }
  }
#pragma unroll
  for (int w = 8; w > 0; w >>= 1)
#pragma unroll
    for (int j = 0; j < w; ++j) lanes[j] = __fadd_rn(lanes[j], lanes[j + w]);
  float sum = lanes[0];
  for (; i < dsub; ++i) {
    const float d = __fsub_rn(__ldg(a + i), __ldg(b + i));
    sum = __fadd_rn(sum, __fmul_rn(d, d));
  }
  tables[idx] = sum;
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
int kpw_for(int k) { return k <= 32 ? 1 : k <= 64 ? 2 : k <= 128 ? 4 : 8; }

size_t workspace_for(int64_t n_queries, int64_t n_cand, int k) {
  const int64_t tiles = n_cand > 0 ? (n_cand + kTile - 1) / kTile : 1;
  const size_t kp = size_t(kpw_for(k)) * 32;
  return size_t(n_queries) * size_t(tiles) * kp * 8 + 256;
}

template <int KPW, int QG, typename Kernel, typename... Args>
cudaError_t launch_scan(Kernel kern, int64_t n_queries, int64_t n_tiles,
                        size_t smem, cudaStream_t stream, Args... args) {
  static std::atomic<int> configured[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  if (dev < 0 || dev >= 64 || configured[dev].load() < int(smem)) {
    cudaError_t err = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < 64) configured[dev].store(227 * 1024);
  }
  const int64_t groups = (n_queries + QG - 1) / QG;
  const int64_t blocks = groups * n_tiles;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  kern<<<dim3(unsigned(blocks)), kThreads, smem, stream>>>(args...);
  return cudaGetLastError();
}

template <int KPW>
cudaError_t merge(const float* wd, const uint32_t* wn, const ScanShape& sh,
                  const vectra_scan_results& res, cudaStream_t stream) {
  const int64_t blocks = (sh.n_queries + 3) / 4;
  merge_kernel<KPW><<<dim3(unsigned(blocks)), 128, 0, stream>>>(
      wd, wn, sh, res.distances, res.nodes, res.counts);
  return cudaGetLastError();
}

template <int KPW, int QG>
cudaError_t run_l2(const vectra_scan_l2_args* a, const ScanShape& sh,
                   float* wd, uint32_t* wn, cudaStream_t stream) {
  const int dpad = (a->dimension + 3) & ~3;
  const size_t smem = size_t(QG) * dpad * 4 + size_t(QG) * kWarps * KPW * 32 * 8;
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  const int vec4 = (a->dimension % 4 == 0) && (a->row_stride % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(a->rows) % 16 == 0);
  cudaError_t err = launch_scan<KPW, QG>(
      l2_scan_kernel<KPW, QG>, sh.n_queries, sh.n_tiles, smem, stream,
      a->queries, a->query_stride, a->rows, a->row_stride, a->dimension, vec4,
      sh, wd, wn);
  if (err != cudaSuccess) return err;
  return merge<KPW>(wd, wn, sh, a->results, stream);
}

template <int KPW, int QG>
cudaError_t run_pq(const vectra_scan_pq_args* a, const ScanShape& sh,
                   float* wd, uint32_t* wn, cudaStream_t stream) {
  const size_t smem = size_t(QG) * a->subspaces * VECTRA_PQ_CENTROIDS * 4 +
                      size_t(QG) * kWarps * KPW * 32 * 8;
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  const int vec16 = (a->subspaces % 16 == 0) && (a->code_stride % 16 == 0) &&
                    (reinterpret_cast<uintptr_t>(a->codes) % 16 == 0);
  cudaError_t err = launch_scan<KPW, QG>(
      pq_scan_kernel<KPW, QG>, sh.n_queries, sh.n_tiles, smem, stream,
      a->tables, a->codes, a->code_stride, a->subspaces, vec16, sh, wd, wn);
  if (err != cudaSuccess) return err;
  return merge<KPW>(wd, wn, sh, a->results, stream);
}

// Queries per CTA: 8 (or the most that fit beside the per-warp lists) for
// scans of every row; 1 for per-query candidate lists.
template <typename Run>
cudaError_t by_kpw(int k, bool shared_candidates, int per_query_floats,
                   Run run) {
  const int kpw = kpw_for(k);
  auto fits = [&](int qg) {
    return size_t(qg) * per_query_floats * 4 + size_t(qg) * kWarps * kpw * 32 * 8 <=
           size_t(200) * 1024;
  };
  const int qg = !shared_candidates ? 1
                 : (kpw <= 2 && fits(8)) ? 8
                 : (kpw <= 4 && fits(4)) ? 4
                 : fits(2) ? 2 : 1;
  switch (kpw) {
    case 1:
      return qg == 8 ? run.template go<1, 8>() : qg == 4 ? run.template go<1, 4>()
           : qg == 2 ? run.template go<1, 2>() : run.template go<1, 1>();
    case 2:
      return qg == 8 ? run.template go<2, 8>() : qg == 4 ? run.template go<2, 4>()
           : qg == 2 ? run.template go<2, 2>() : run.template go<2, 1>();
    case 4:
      return qg >= 4 ? run.template go<4, 4>() : qg == 2 ? run.template go<4, 2>()
           : run.template go<4, 1>();
    default:
      return qg >= 2 ? run.template go<8, 2>() : run.template go<8, 1>();
  }
}

struct L2Run {
  const vectra_scan_l2_args* a;
  const ScanShape* sh;
  float* wd;
  uint32_t* wn;
  cudaStream_t stream;
  template <int KPW, int QG>
  cudaError_t go() const { return run_l2<KPW, QG>(a, *sh, wd, wn, stream); }
};
struct PqRun {
  const vectra_scan_pq_args* a;
  const ScanShape* sh;
  float* wd;
  uint32_t* wn;
  cudaStream_t stream;
  template <int KPW, int QG>
  cudaError_t go() const { return run_pq<KPW, QG>(a, *sh, wd, wn, stream); }
};

// Common argument checks and workspace layout: (distances | nodes).
int prepare(int64_t n_queries, int64_t n_rows, int k,
            const vectra_scan_candidates& cand,
            const vectra_scan_results& res, void* workspace,
            size_t workspace_bytes, ScanShape* sh,
            float** wd, uint32_t** wn) {
  if (res.distances == nullptr || res.nodes == nullptr) return VECTRA_ERR_NULL;
  if (n_queries < 0 || n_rows < 0 || n_rows >= 0xffffffffLL)
    return VECTRA_ERR_SHAPE;
  if (k < 1 || k > VECTRA_SCAN_MAX_K) return VECTRA_ERR_UNSUPPORTED;
  if (cand.offsets != nullptr &&
      (cand.ids == nullptr || cand.max_per_query < 0))
    return VECTRA_ERR_NULL;
  const int64_t nc = cand.offsets == nullptr ? n_rows : cand.max_per_query;
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 15) ||
      workspace_bytes < workspace_for(n_queries, nc, k))
    return VECTRA_ERR_NULL;
  sh->n_queries = n_queries;
  sh->n_rows = n_rows;
  sh->n_tiles = nc > 0 ? (nc + kTile - 1) / kTile : 1;
  sh->offsets = cand.offsets;
  sh->ids = cand.ids;
  sh->k = k;
  const size_t entries =
      size_t(n_queries) * size_t(sh->n_tiles) * size_t(kpw_for(k)) * 32;
  *wd = static_cast<float*>(workspace);
  *wn = reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) +
                                    ((entries * 4 + 15) & ~size_t(15)));
  return VECTRA_OK;
}

}  // namespace
}  // namespace scan
}  // namespace vectra

using namespace vectra::scan;  // NOLINT

extern "C" {

VECTRA_API size_t vectra_scan_workspace_bytes(int64_t n_queries,
                                              int64_t max_candidates,
                                              int32_t k) {
  if (n_queries < 0 || max_candidates < 0 || k < 1 || k > VECTRA_SCAN_MAX_K)
    return 0;
  return workspace_for(n_queries, max_candidates, k);
}

VECTRA_API int vectra_scan_l2_topk(const vectra_scan_l2_args* a,
                                   void* stream) {
  if (a == nullptr || a->queries == nullptr || a->rows == nullptr)
    return VECTRA_ERR_NULL;
  if (a->dimension < 1 || a->dimension > 4096 ||
      a->query_stride < a->dimension || a->row_stride < a->dimension)
    return VECTRA_ERR_SHAPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ScanShape sh;
  float* wd;
  uint32_t* wn;
  const int st = prepare(a->n_queries, a->n_rows, a->k, a->candidates,
                         a->results, a->workspace, a->workspace_bytes, &sh,
                         &wd, &wn);
  if (st != VECTRA_OK) return st;
  if (a->n_queries == 0) return VECTRA_OK;
  const int dpad = (a->dimension + 3) & ~3;
  L2Run run{a, &sh, wd, wn, s};
  return by_kpw(a->k, a->candidates.offsets == nullptr, dpad, run) ==
                 cudaSuccess
             ? VECTRA_OK
             : VECTRA_ERR_CUDA;
}

VECTRA_API int vectra_scan_pq_topk(const vectra_scan_pq_args* a,
                                   void* stream) {
  if (a == nullptr || a->tables == nullptr || a->codes == nullptr)
    return VECTRA_ERR_NULL;
  if (a->subspaces < 1 || a->subspaces > VECTRA_SCAN_MAX_SUBSPACES ||
      a->code_stride < a->subspaces)
    return VECTRA_ERR_SHAPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ScanShape sh;
  float* wd;
  uint32_t* wn;
  const int st = prepare(a->n_queries, a->n_rows, a->k, a->candidates,
                         a->results, a->workspace, a->workspace_bytes, &sh,
                         &wd, &wn);
  if (st != VECTRA_OK) return st;
  if (a->n_queries == 0) return VECTRA_OK;
  PqRun run{a, &sh, wd, wn, s};
  return by_kpw(a->k, a->candidates.offsets == nullptr,
                a->subspaces * VECTRA_PQ_CENTROIDS, run) == cudaSuccess
             ? VECTRA_OK
             : VECTRA_ERR_CUDA;
}

VECTRA_API int vectra_pq_distance_tables(const float* queries,
                                         int64_t n_queries,
                                         int64_t query_stride,
                                         const float* codebooks,
                                         int32_t dimension, int32_t subspaces,
                                         float* tables, void* stream) {
  if (queries == nullptr || codebooks == nullptr || tables == nullptr)
    return VECTRA_ERR_NULL;
  if (n_queries < 0 || dimension < 1 || subspaces < 1 ||
      subspaces > VECTRA_SCAN_MAX_SUBSPACES || dimension % subspaces != 0 ||
      query_stride < dimension)
    return VECTRA_ERR_SHAPE;
  const int64_t total = n_queries * subspaces * VECTRA_PQ_CENTROIDS;
  if (total == 0) return VECTRA_OK;
  const int64_t blocks = (total + 255) / 256;
  pq_tables_kernel<<<dim3(unsigned(blocks)), 256, 0,
                     static_cast<cudaStream_t>(stream)>>>(
      queries, n_queries, query_stride, codebooks, dimension / subspaces,
      subspaces, tables);
  return cudaGetLastError() == cudaSuccess ? VECTRA_OK : VECTRA_ERR_CUDA;
}

}  // extern "C"
