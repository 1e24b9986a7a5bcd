// scan.cu: exhaustive top-k scans of an index shard (include/vectra_scan.h),
// the GPU counterparts of the reference engine's candidate scoring:
// ShardIndex::ExhaustiveSearch (engine/src/index/shard_index.cc:236-266),
// L2SquaredDistance / PqAdcDistance (engine/src/index/simd_distance.cc) and
// ProductQuantizer::ComputeDistanceTable (engine/src/index/pq_codec.cc).
//
// Design (B200):
//  * Candidates are scanned in tiles of kTile = 4,096 by persistent CTAs of
//    8 warps: for a group of QG queries (their vectors, or their PQ tables,
//    in shared memory) a CTA takes tiles slot, slot + n_slots, ... (about
//    two CTAs per SM over all groups). The CTAs of all query groups with the
//    same slot run together and read each tile from HBM once (L2 serves
//    the others).
//  * An admission bound first: a sample pass scans each query's first tile
//    and its k-th nearest there bounds the true k-th nearest from above
//    (as a (distance, node) pair), so the main pass offers a warp's list
//    only the candidates at or under it (about k of every tile's 4,096);
//    without it every warp list would be filled from empty and insertions,
//    not distances, would dominate.
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

#include <algorithm>
#include <atomic>
#include <mutex>
#include <utility>
#include <vector>

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
  int64_t scan_tiles;     // tiles this launch scans (n_tiles, or 1: sample)
  int64_t n_slots;        // CTAs (and partial lists) per query group
  const int64_t* offsets;  // per-query candidates (CSR), or null
  const uint32_t* ids;
  const float* bound_d;   // per-query admission bound, or null
  const uint32_t* bound_n;
  float* sample_out;      // sample mode: per-query bound to lower, or null
  int k;
};

// Lowers *addr to v (atomically, float order).
__device__ __forceinline__ void atomic_min_float(float* addr, float v) {
  if (!(v == v)) return;  // NaN
  unsigned int* a = reinterpret_cast<unsigned int*>(addr);
  unsigned int old = *a, assumed;
  do {
    assumed = old;
    if (__uint_as_float(assumed) <= v) return;
    old = atomicCAS(a, assumed, __float_as_uint(v));
  } while (old != assumed);
}

// Sample mode: each lane's minimum distance over its rows of the tile; the
// k-th smallest of the CTA's 256 lane minima bounds the tile's k-th nearest
// from above (at least k rows are at or under it), and the smallest such
// bound over the sampled tiles bounds the scan's. `mins` are per query.
template <int QG>
__device__ __forceinline__ void sample_bound(const float (&mins)[QG],
                                             float* sbuf, int64_t q0,
                                             const ScanShape& sh) {
  const int t = threadIdx.x;
#pragma unroll
  for (int g = 0; g < QG; ++g) sbuf[g * kThreads + t] = mins[g];
  __syncthreads();
  // Bitonic sort of each query's 256 minima, ascending.
  for (int size = 2; size <= kThreads; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const int partner = t ^ stride;
      if (partner > t) {
        const bool up = (t & size) == 0;
#pragma unroll
        for (int g = 0; g < QG; ++g) {
          float& a = sbuf[g * kThreads + t];
          float& b = sbuf[g * kThreads + partner];
          if ((a > b) == up) {
            const float x = a;
            a = b;
            b = x;
          }
        }
      }
      __syncthreads();
    }
  }
  if (t < QG && q0 + t < sh.n_queries)
    atomic_min_float(sh.sample_out + q0 + t,
                     sbuf[t * kThreads + (sh.k - 1 < kThreads ? sh.k - 1
                                                                : kThreads - 1)]);
}

// The admission bound of query q: candidates farther than it are not
// offered (+inf / no bound when absent).
__device__ __forceinline__ void bound_of(const ScanShape& sh, int64_t q,
                                         float& bd, uint32_t& bn) {
  if (sh.bound_d != nullptr && q < sh.n_queries) {
    bd = sh.bound_d[q];
    bn = sh.bound_n[q];
  } else {
    bd = INFINITY;
    bn = kNoNode;
  }
}

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
                                           int64_t q0, int64_t nq, int64_t slot,
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
    const size_t base = (size_t(q0 + g) * sh.n_slots + slot) * KP;
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
                   int dim, int vec4, float* wd, uint32_t* wn, ScanShape sh) {
  extern __shared__ __align__(16) float smem_f[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_groups = (sh.n_queries + QG - 1) / QG;
  const int64_t group = blockIdx.x % n_groups;
  const int64_t slot = blockIdx.x / n_groups;
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
  float bd[QG];
  uint32_t bn[QG];
  float mins[QG];
  const bool sampling = sh.sample_out != nullptr;
#pragma unroll
  for (int g = 0; g < QG; ++g) {
    lists[g].clear();
    bound_of(sh, q0 + g, bd[g], bn[g]);
    mins[g] = INFINITY;
  }
  for (int64_t tile = slot; tile < sh.scan_tiles; tile += sh.n_slots)
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
        // Eight 16-byte loads of the row in flight before any is used.
        constexpr int kBatch = 8;
        int c = 0;
        for (; c + 4 * kBatch <= dim; c += 4 * kBatch) {
          float4 rv[kBatch];
#pragma unroll
          for (int b = 0; b < kBatch; ++b)
            rv[b] = __ldg(reinterpret_cast<const float4*>(row + c + 4 * b));
#pragma unroll
          for (int b = 0; b < kBatch; ++b) {
            const uint64_t r01 = pk(rv[b].x, rv[b].y);
            const uint64_t r23 = pk(rv[b].z, rv[b].w);
#pragma unroll
            for (int g = 0; g < QG; ++g) {
              const float4 qv = *reinterpret_cast<const float4*>(
                  sq + g * dpad + c + 4 * b);
              const uint64_t d01 = sub2(pk(qv.x, qv.y), r01);
              const uint64_t d23 = sub2(pk(qv.z, qv.w), r23);
              acc[g][0] = fma2(d01, d01, acc[g][0]);
              acc[g][1] = fma2(d23, d23, acc[g][1]);
            }
          }
        }
        for (; c < dim; c += 4) {
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
    if (sampling) {
#pragma unroll
      for (int g = 0; g < QG; ++g) mins[g] = fminf(mins[g], dist[g]);
      continue;
    }
#pragma unroll
    for (int g = 0; g < QG; ++g) {
      const bool admit = !closer(bd[g], bn[g], dist[g], node);
      lists[g].offer(admit ? dist[g] : INFINITY, admit ? node : kNoNode,
                     sh.k, lane);
    }
  }
  if (sampling) {
    sample_bound<QG>(mins, sd, q0, sh);
    return;
  }
  merge_tile<KPW, QG>(lists, sd, sn, q0, sh.n_queries, slot, sh, wd, wn);
}

// ---------------------------------------------------------------------------
// PQ (asymmetric distance) scan.
// ---------------------------------------------------------------------------
// The sum of table entries for one code in PqAdcDistance's order; MS > 0:
// MS sub-spaces known at compile time (code bytes in registers).
template <int MS>
__device__ __forceinline__ float adc_sum(const float* t, const uint8_t* code,
                                         int m) {
  float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
  const int mm = MS > 0 ? MS : m;
  int s = 0;
#pragma unroll
  for (; s + 4 <= mm; s += 4) {
    l0 = __fadd_rn(l0, t[(s + 0) * 256 + code[s + 0]]);
    l1 = __fadd_rn(l1, t[(s + 1) * 256 + code[s + 1]]);
    l2 = __fadd_rn(l2, t[(s + 2) * 256 + code[s + 2]]);
    l3 = __fadd_rn(l3, t[(s + 3) * 256 + code[s + 3]]);
  }
  float sum = __fadd_rn(__fadd_rn(l0, l1), __fadd_rn(l2, l3));
#pragma unroll
  for (; s < mm; ++s) sum = __fadd_rn(sum, t[s * 256 + code[s]]);
  return sum;
}

template <int KPW, int QG, int MS>
__global__ void __launch_bounds__(kThreads)
    pq_scan_kernel(const float* __restrict__ tables,
                   const uint8_t* __restrict__ codes, int64_t code_stride,
                   int m, int vec16, float* wd, uint32_t* wn, ScanShape sh) {
  extern __shared__ __align__(16) float smem_f[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_groups = (sh.n_queries + QG - 1) / QG;
  const int64_t group = blockIdx.x % n_groups;
  const int64_t slot = blockIdx.x / n_groups;
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
  float bd[QG];
  uint32_t bn[QG];
  float mins[QG];
  const bool sampling = sh.sample_out != nullptr;
#pragma unroll
  for (int g = 0; g < QG; ++g) {
    lists[g].clear();
    bound_of(sh, q0 + g, bd[g], bn[g]);
    mins[g] = INFINITY;
  }
  constexpr int kCodeBytes = MS > 0 ? MS : VECTRA_SCAN_MAX_SUBSPACES;
  for (int64_t tile = slot; tile < sh.scan_tiles; tile += sh.n_slots)
  for (int r = 0; r < kRowsPerLane; ++r) {
    const int64_t i = tile * kTile + (int64_t(r) * kWarps + warp) * 32 + lane;
    const uint32_t node = candidate(sh, q0, i);
    float dist[QG];
    if (node != kNoNode) {
      const uint8_t* cp = codes + int64_t(node) * code_stride;
      // The code: in registers when MS is known (16-byte loads), else in a
      // local array.
      union {
        uint4 w[(kCodeBytes + 15) / 16];
        uint8_t b[((kCodeBytes + 15) / 16) * 16];
      } code;
      if (MS > 0 && vec16) {
#pragma unroll
        for (int i = 0; i < (kCodeBytes + 15) / 16; ++i)
          code.w[i] = __ldg(reinterpret_cast<const uint4*>(cp) + i);
      } else {
        for (int s = 0; s < m; ++s) code.b[s] = __ldg(cp + s);
      }
#pragma unroll
      for (int g = 0; g < QG; ++g)
        // PqAdcDistance (simd_distance.cc:71-85): four chains, then the
        // tail, in this order.
        dist[g] = adc_sum<MS>(st + g * tsz, code.b, m);
    } else {
#pragma unroll
      for (int g = 0; g < QG; ++g) dist[g] = INFINITY;
    }
    if (sampling) {
#pragma unroll
      for (int g = 0; g < QG; ++g) mins[g] = fminf(mins[g], dist[g]);
      continue;
    }
#pragma unroll
    for (int g = 0; g < QG; ++g) {
      const bool admit = !closer(bd[g], bn[g], dist[g], node);
      lists[g].offer(admit ? dist[g] : INFINITY, admit ? node : kNoNode,
                     sh.k, lane);
    }
  }
  if (sampling) {
    sample_bound<QG>(mins, sd, q0, sh);
    return;
  }
  merge_tile<KPW, QG>(lists, sd, sn, q0, sh.n_queries, slot, sh, wd, wn);
}

// ---------------------------------------------------------------------------
// Merge of a query's tiles: one warp per query.
// ---------------------------------------------------------------------------
template <int KPW>
__global__ void __launch_bounds__(kThreads)
    merge_kernel(const float* wd, const uint32_t* wn, ScanShape sh,
                 float* out_d, uint32_t* out_n, int32_t* counts) {
  // One CTA per query: warp w merges slots w, w + 8, ... (the next batch's
  // loads issued before the current batch is offered); warp 0 merges the
  // eight lists.
  __shared__ float md[kWarps * KPW * 32];
  __shared__ uint32_t mn[kWarps * KPW * 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t q = blockIdx.x;
  constexpr int KP = KPW * 32;
  const int k = sh.k;
  const size_t base = size_t(q) * sh.n_slots * KP;
  WarpList<KPW> m;
  m.clear();
  const int64_t per_warp = (sh.n_slots + kWarps - 1 - warp) / kWarps;
  const int64_t n_batches = per_warp * KPW;  // 32 entries per batch
  auto at = [&](int64_t b) {  // entry of batch b for this lane
    const int64_t slot = warp + (b / KPW) * kWarps;
    return base + size_t(slot) * KP + (b % KPW) * 32 + lane;
  };
  float nd = INFINITY;
  uint32_t nn = kNoNode;
  if (n_batches > 0) {
    nd = wd[at(0)];
    nn = wn[at(0)];
  }
  for (int64_t b = 0; b < n_batches; ++b) {
    const float cd = nd;
    const uint32_t cn = nn;
    if (b + 1 < n_batches) {
      nd = wd[at(b + 1)];
      nn = wn[at(b + 1)];
    }
    m.offer(cd, cn, k, lane);
  }
#pragma unroll
  for (int s = 0; s < KPW; ++s) {
    md[warp * KP + s * 32 + lane] = m.d[s];
    mn[warp * KP + s * 32 + lane] = m.n[s];
  }
  __syncthreads();
  if (warp != 0) return;
  for (int i = KP; i < kWarps * KP; i += 32) m.offer(md[i + lane], mn[i + lane], k, lane);
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

// Admission bounds start open: (+inf, no node); the sample pass lowers the
// distances, and the node stays kNoNode (every distance at or under the
// bound is admitted).
__global__ void bound_init_kernel(int64_t nq, float* bound_d,
                                  uint32_t* bound_n) {
  const int64_t q = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  bound_d[q] = INFINITY;
  bound_n[q] = kNoNode;
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

// Partial lists per query group at most (the main pass's CTAs per group).
constexpr int64_t kMaxSlots = 512;
// Tiles the sample pass bounds the scan from.
constexpr int64_t kSampleTiles = 16;

int64_t tiles_for(int64_t n_cand) {
  return n_cand > 0 ? (n_cand + kTile - 1) / kTile : 1;
}

// Workspace: partial lists [n_queries][slots][32 KPW] of distances, then of
// nodes, then the admission bounds (distances, nodes) [n_queries].
size_t workspace_for(int64_t n_queries, int64_t n_cand, int k) {
  const int64_t slots = std::min(tiles_for(n_cand), kMaxSlots);
  const size_t kp = size_t(kpw_for(k)) * 32;
  const size_t lists = size_t(n_queries) * size_t(slots) * kp;
  return ((lists * 4 + 15) & ~size_t(15)) * 2 + size_t(n_queries) * 8 + 256;
}

struct Workspace {
  float* wd;
  uint32_t* wn;
  float* bound_d;
  uint32_t* bound_n;
};

// Sets a kernel's dynamic shared-memory limit once per (kernel, device).
// (Instantiations that differ only in template values share a function
// pointer type, so the record is kept by address.)
cudaError_t allow_smem(const void* kern) {
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& e : done)
    if (e.first == kern && e.second == dev) return cudaSuccess;
  cudaError_t err = cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (err == cudaSuccess) done.emplace_back(kern, dev);
  return err;
}

template <int KPW, int QG, typename Kernel, typename... Args>
cudaError_t launch_scan(Kernel kern, const ScanShape& sh, size_t smem,
                        cudaStream_t stream, Args... args) {
  cudaError_t err = allow_smem(reinterpret_cast<const void*>(kern));
  if (err != cudaSuccess) return err;
  const int64_t groups = (sh.n_queries + QG - 1) / QG;
  const int64_t blocks = groups * sh.n_slots;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  kern<<<dim3(unsigned(blocks)), kThreads, smem, stream>>>(args..., sh);
  return cudaGetLastError();
}

template <int KPW>
cudaError_t merge(const Workspace& w, const ScanShape& sh,
                  const vectra_scan_results& res, cudaStream_t stream) {
  merge_kernel<KPW><<<dim3(unsigned(sh.n_queries)), kThreads, 0, stream>>>(
      w.wd, w.wn, sh, res.distances, res.nodes, res.counts);
  return cudaGetLastError();
}

// The scan in four launches when the candidates span several tiles: the
// sample pass over each query's first tile (one slot), its admission
// bounds, the main pass with them, and the merge of the main pass's lists.
template <int KPW, int QG, typename Launch>
cudaError_t scan_passes(const ScanShape& base, const Workspace& w,
                        const vectra_scan_results& res, cudaStream_t stream,
                        Launch launch) {
  ScanShape sh = base;
  sh.bound_d = nullptr;
  sh.bound_n = nullptr;
  sh.sample_out = nullptr;
  if (base.n_tiles > 1) {
    // Bounds from the first kSampleTiles tiles, one CTA each.
    const int64_t nb = (sh.n_queries + 127) / 128;
    bound_init_kernel<<<dim3(unsigned(nb)), 128, 0, stream>>>(
        sh.n_queries, w.bound_d, w.bound_n);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    sh.scan_tiles = std::min(base.n_tiles, kSampleTiles);
    sh.n_slots = sh.scan_tiles;
    sh.sample_out = w.bound_d;
    if ((err = launch(sh)) != cudaSuccess) return err;
    sh.sample_out = nullptr;
    sh.bound_d = w.bound_d;
    sh.bound_n = w.bound_n;
  }
  const int64_t groups = (sh.n_queries + QG - 1) / QG;
  int64_t slots = (2 * int64_t(device_sm_count()) + groups - 1) / groups;
  slots = std::max<int64_t>(1, std::min({slots, base.n_tiles, kMaxSlots}));
  sh.scan_tiles = base.n_tiles;
  sh.n_slots = slots;
  cudaError_t err = launch(sh);
  if (err != cudaSuccess) return err;
  return merge<KPW>(w, sh, res, stream);
}

template <int KPW, int QG>
cudaError_t run_l2(const vectra_scan_l2_args* a, const ScanShape& sh,
                   const Workspace& w, cudaStream_t stream) {
  const int dpad = (a->dimension + 3) & ~3;
  const size_t smem = size_t(QG) * dpad * 4 + size_t(QG) * kWarps * KPW * 32 * 8;
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  const int vec4 = (a->dimension % 4 == 0) && (a->row_stride % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(a->rows) % 16 == 0);
  return scan_passes<KPW, QG>(sh, w, a->results, stream,
                              [&](const ScanShape& s2) {
    return launch_scan<KPW, QG>(l2_scan_kernel<KPW, QG>, s2, smem, stream,
                                a->queries, a->query_stride, a->rows,
                                a->row_stride, a->dimension, vec4, w.wd,
                                w.wn);
  });
}

template <int KPW, int QG>
cudaError_t run_pq(const vectra_scan_pq_args* a, const ScanShape& sh,
                   const Workspace& w, cudaStream_t stream) {
  const size_t smem = size_t(QG) * a->subspaces * VECTRA_PQ_CENTROIDS * 4 +
                      size_t(QG) * kWarps * KPW * 32 * 8;
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  const int vec16 = (a->subspaces % 16 == 0) && (a->code_stride % 16 == 0) &&
                    (reinterpret_cast<uintptr_t>(a->codes) % 16 == 0);
  auto kernel = a->subspaces == 16 && vec16   ? pq_scan_kernel<KPW, QG, 16>
                : a->subspaces == 8 && a->code_stride % 16 == 0 &&
                          reinterpret_cast<uintptr_t>(a->codes) % 16 == 0
                    ? pq_scan_kernel<KPW, QG, 8>
                : a->subspaces == 32 && vec16 ? pq_scan_kernel<KPW, QG, 32>
                : a->subspaces == 64 && vec16 ? pq_scan_kernel<KPW, QG, 64>
                                              : pq_scan_kernel<KPW, QG, 0>;
  const int vec_ok = a->subspaces == 8 ? (a->code_stride % 16 == 0 &&
                                          reinterpret_cast<uintptr_t>(
                                              a->codes) % 16 == 0)
                                       : vec16;
  return scan_passes<KPW, QG>(sh, w, a->results, stream,
                              [&](const ScanShape& s2) {
    return launch_scan<KPW, QG>(kernel, s2, smem, stream, a->tables, a->codes,
                                a->code_stride, a->subspaces, vec_ok, w.wd,
                                w.wn);
  });
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
  const Workspace* w;
  cudaStream_t stream;
  template <int KPW, int QG>
  cudaError_t go() const { return run_l2<KPW, QG>(a, *sh, *w, stream); }
};
struct PqRun {
  const vectra_scan_pq_args* a;
  const ScanShape* sh;
  const Workspace* w;
  cudaStream_t stream;
  template <int KPW, int QG>
  cudaError_t go() const { return run_pq<KPW, QG>(a, *sh, *w, stream); }
};

// Common argument checks and the workspace layout.
int prepare(int64_t n_queries, int64_t n_rows, int k,
            const vectra_scan_candidates& cand,
            const vectra_scan_results& res, void* workspace,
            size_t workspace_bytes, ScanShape* sh, Workspace* w) {
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
  sh->n_tiles = tiles_for(nc);
  sh->scan_tiles = sh->n_tiles;
  sh->n_slots = 1;
  sh->offsets = cand.offsets;
  sh->ids = cand.ids;
  sh->bound_d = nullptr;
  sh->bound_n = nullptr;
  sh->k = k;
  const size_t lists = size_t(n_queries) *
                       size_t(std::min(sh->n_tiles, kMaxSlots)) *
                       size_t(kpw_for(k)) * 32;
  const size_t bytes = (lists * 4 + 15) & ~size_t(15);
  char* base = static_cast<char*>(workspace);
  w->wd = reinterpret_cast<float*>(base);
  w->wn = reinterpret_cast<uint32_t*>(base + bytes);
  w->bound_d = reinterpret_cast<float*>(base + 2 * bytes);
  w->bound_n = reinterpret_cast<uint32_t*>(base + 2 * bytes +
                                           size_t(n_queries) * 4);
  return VECTRA_OK;
}

}  // namespace
}  // namespace scan
}  // namespace vectra

// Scratch of vectra_scan_l2_topk_noalloc, for callers that cannot allocate:
// one array per device context in the module's global memory, held until
// the process exits. In host code its name is only a stand-in; the device
// address is looked up once per device (cudaGetSymbolAddress, that device
// current) and passed to the kernels. Calls on one device take turns with
// it (an event per device), since overlapping calls would race on it.
static __device__ __align__(256) unsigned char
    g_scan_scratch[size_t(VECTRA_SCAN_NOALLOC_SCRATCH_BYTES)];

namespace vectra {
namespace scan {
namespace {

struct StaticScratch {
  void* ptr = nullptr;
  cudaEvent_t last_use = nullptr;  // the previous call's work on it
};

std::mutex g_scratch_mu;
StaticScratch g_scratch[64];

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
  Workspace w;
  const int st = prepare(a->n_queries, a->n_rows, a->k, a->candidates,
                         a->results, a->workspace, a->workspace_bytes, &sh,
                         &w);
  if (st != VECTRA_OK) return st;
  if (a->n_queries == 0) return VECTRA_OK;
  const int dpad = (a->dimension + 3) & ~3;
  L2Run run{a, &sh, &w, s};
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
  Workspace w;
  const int st = prepare(a->n_queries, a->n_rows, a->k, a->candidates,
                         a->results, a->workspace, a->workspace_bytes, &sh,
                         &w);
  if (st != VECTRA_OK) return st;
  if (a->n_queries == 0) return VECTRA_OK;
  PqRun run{a, &sh, &w, s};
  return by_kpw(a->k, a->candidates.offsets == nullptr,
                a->subspaces * VECTRA_PQ_CENTROIDS, run) == cudaSuccess
             ? VECTRA_OK
             : VECTRA_ERR_CUDA;
}

VECTRA_API int vectra_scan_l2_topk_noalloc(const vectra_scan_l2_args* a,
                                           void* stream) {
  if (a == nullptr) return VECTRA_ERR_NULL;
  if (a->k < 1 || a->k > VECTRA_SCAN_MAX_K) return VECTRA_ERR_UNSUPPORTED;
  const int64_t nc = a->candidates.offsets == nullptr
                         ? a->n_rows
                         : a->candidates.max_per_query;
  if (a->n_queries < 0 || nc < 0) return VECTRA_ERR_SHAPE;
  if (workspace_for(a->n_queries, nc, a->k) >
      size_t(VECTRA_SCAN_NOALLOC_SCRATCH_BYTES))
    return VECTRA_ERR_UNSUPPORTED;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return VECTRA_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  StaticScratch& ss = g_scratch[dev];
  if (ss.ptr == nullptr) {
    if (cudaGetSymbolAddress(&ss.ptr, g_scan_scratch) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.last_use, cudaEventDisableTiming) !=
            cudaSuccess) {
      ss.ptr = nullptr;
      return VECTRA_ERR_CUDA;
    }
  }
  vectra_scan_l2_args b = *a;
  b.workspace = ss.ptr;
  b.workspace_bytes = size_t(VECTRA_SCAN_NOALLOC_SCRATCH_BYTES);
  // After the previous call's kernels, whatever stream they ran on.
  if (cudaStreamWaitEvent(s, ss.last_use, 0) != cudaSuccess)
    return VECTRA_ERR_CUDA;
  const int status = vectra_scan_l2_topk(&b, stream);
  if (cudaEventRecord(ss.last_use, s) != cudaSuccess) return VECTRA_ERR_CUDA;
  return status;
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
