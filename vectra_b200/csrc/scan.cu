// scan.cu: exhaustive top-k scans of an index shard (include/vectra_scan.h),
// the GPU counterparts of the reference engine's candidate scoring:
// ShardIndex::ExhaustiveSearch (engine/src/index/shard_index.cc:236-266),
// L2SquaredDistance / PqAdcDistance (engine/src/index/simd_distance.cc) and
// ProductQuantizer::ComputeDistanceTable (engine/src/index/pq_codec.cc).
//
// Design (B200): score every candidate once at HBM speed, keep almost none.
//  * Distances: QG queries per CTA, a lane per candidate row (PQ tables or
//    query vectors in shared memory), or for L2 over every row 16 lanes per
//    row staged by bulk copy (l2_bulk_kernel below). L2 sums (q_d - r_d)^2
//    in float32 with packed f32x2 subtract/FMA; PQ sums table entries
//    in PqAdcDistance's order (four chains, (l0 + l1) + (l2 + l3), then the
//    tail: bit-identical to the reference). A distance becomes a 32-bit key
//    whose unsigned order is the float order, and (key, node) as one 64-bit
//    value orders candidates as CloserFirst does (distance, then node id;
//    engine/include/vectra/index/search_scratch.h:35-40).
//  * Levels. Level 0 scores a spread sample (groups of 32 consecutive
//    candidates, evenly spaced) and stores every key; a select kernel finds
//    its k-th smallest key, an upper bound on the true k-th distance (at
//    least k candidates are at or under it). Each further level scores a
//    larger sample, or at last every candidate, and appends only the
//    candidates at or under the current bound to a per-query buffer (a
//    ballot and one atomic per warp); its select lowers the bound again.
//    Sample sizes are planned so that the last level admits a few thousand
//    candidates per query out of millions.
//  * Select: one CTA of 1,024 threads per query stages the buffer's keys in
//    shared memory; one histogram over their range (2,048 bins) usually
//    leaves few enough entries at or under the bin of the k-th to sort
//    (bitonic: one warp in registers up to 128 entries, in shared memory up
//    to 256, the block up to 2,048); otherwise a radix select over 11-bit
//    digits of (key, node) narrows them first. A bound needs only the end
//    of the k-th's bin.
//  * A last level that admits more candidates than its buffer holds (mass
//    ties at the bound) is redone for that query by the warp-list scan:
//    per-warp sorted lists in registers fed by ballot-filtered insertion,
//    merged per tile and per query: exact for any input, slower.
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>
#include <utility>
#include <vector>

#include "rbf_common.cuh"
#include "vectra_scan.h"

namespace vectra {
namespace scan {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxRowsPerLane = 16;
constexpr int kListTile = kThreads * kMaxRowsPerLane;  // warp-list scan tile
constexpr uint32_t kNoNode = 0xffffffffu;
constexpr uint32_t kNoBound = 0xffffffffu;  // admits every key
constexpr unsigned kFull = 0xffffffffu;
// Candidate buffer per query (entries), and the select kernel's shape.
constexpr int64_t kCap = 32768;
constexpr int kSelThreads = 1024;
constexpr int kSortMax = 2048;
// Candidates scored by level 0 when a query has more than kCap.
constexpr int64_t kSample0 = 8192;

// Unsigned order of the key = float order of the distance (-0 as +0, NaN
// last).
__device__ __forceinline__ uint32_t dist_key(float d) {
  if (d != d) return 0xffffffffu;
  uint32_t u = __float_as_uint(d);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_dist(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7fffffffu) : ~key);
}

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

// ---------------------------------------------------------------------------
// Scorers: a CTA's queries in shared memory, and their distances to a row.
// ---------------------------------------------------------------------------
template <int QG>
struct L2Score {
  const float* queries;
  int64_t query_stride;
  const float* rows;
  int64_t row_stride;
  int dim;
  int vec4;  // rows 16-byte aligned with dim % 4 == 0

  static size_t smem_floats(int dim) { return size_t(QG) * ((dim + 3) & ~3); }
  __device__ __forceinline__ int floats() const { return QG * ((dim + 3) & ~3); }

  __device__ __forceinline__ void load(float* s, int64_t q0,
                                       int64_t nq) const {
    const int dpad = (dim + 3) & ~3;
    for (int i = threadIdx.x; i < QG * dpad; i += blockDim.x) {
      const int g = i / dpad, c = i - g * dpad;
      s[i] = (q0 + g < nq && c < dim) ? queries[(q0 + g) * query_stride + c]
                                      : 0.f;
    }
  }

  __device__ __forceinline__ void score(const float* sq, uint32_t node,
                                        float (&dist)[QG]) const {
    const int dpad = (dim + 3) & ~3;
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
            const float4 qv =
                *reinterpret_cast<const float4*>(sq + g * dpad + c + 4 * b);
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
      // Element pairs (c, c + 1) in one packed accumulator; an odd last
      // element in the other.
      int c = 0;
      for (; c + 2 <= dim; c += 2) {
        const float r0 = __ldg(row + c), r1 = __ldg(row + c + 1);
#pragma unroll
        for (int g = 0; g < QG; ++g) {
          const uint64_t dd =
              pk(sq[g * dpad + c] - r0, sq[g * dpad + c + 1] - r1);
          acc[g][0] = fma2(dd, dd, acc[g][0]);
        }
      }
      if (c < dim) {
        const float r0 = __ldg(row + c);
#pragma unroll
        for (int g = 0; g < QG; ++g) {
          const uint64_t dd = pk(sq[g * dpad + c] - r0, 0.f);
          acc[g][1] = fma2(dd, dd, acc[g][1]);
        }
      }
    }
#pragma unroll
    for (int g = 0; g < QG; ++g) {
      const float2 a = upk(acc[g][0]), b = upk(acc[g][1]);
      dist[g] = (a.x + a.y) + (b.x + b.y);
    }
  }
};

// The sum of table entries for one code in PqAdcDistance's order
// (simd_distance.cc:71-85): four chains, (l0 + l1) + (l2 + l3), then the
// tail. Code bytes in a local array (any m).
__device__ __forceinline__ float adc_sum_bytes(const float* t,
                                               const uint8_t* code, int m) {
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
  return sum;
}

// The same sum with MS known and the code bytes packed four to a 32-bit
// word (registers).
template <int MS>
__device__ __forceinline__ float adc_sum_words(const float* t,
                                               const uint32_t* w) {
  auto at = [&](int s) {
    return t[s * 256 + ((w[s >> 2] >> ((s & 3) * 8)) & 0xffu)];
  };
  float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
  int s = 0;
#pragma unroll
  for (; s + 4 <= MS; s += 4) {
    l0 = __fadd_rn(l0, at(s + 0));
    l1 = __fadd_rn(l1, at(s + 1));
    l2 = __fadd_rn(l2, at(s + 2));
    l3 = __fadd_rn(l3, at(s + 3));
  }
  float sum = __fadd_rn(__fadd_rn(l0, l1), __fadd_rn(l2, l3));
#pragma unroll
  for (; s < MS; ++s) sum = __fadd_rn(sum, at(s));
  return sum;
}

template <int QG, int MS>
struct PqScore {
  const float* tables;
  const uint8_t* codes;
  int64_t code_stride;
  int m;

  static size_t smem_floats(int m) {
    return size_t(QG) * m * VECTRA_PQ_CENTROIDS;
  }
  __device__ __forceinline__ int floats() const {
    return QG * m * VECTRA_PQ_CENTROIDS;
  }

  __device__ __forceinline__ void load(float* s, int64_t q0,
                                       int64_t nq) const {
    const int tsz = m * VECTRA_PQ_CENTROIDS;
    for (int i = threadIdx.x; i < QG * tsz; i += blockDim.x) {
      const int g = i / tsz;
      s[i] = q0 + g < nq ? tables[(q0 + g) * tsz + (i - g * tsz)] : 0.f;
    }
  }

  // MS > 0 kernels run only on codes whose address and stride are aligned
  // to their 8- or 16-byte loads.
  __device__ __forceinline__ void score(const float* st, uint32_t node,
                                        float (&dist)[QG]) const {
    const int tsz = m * VECTRA_PQ_CENTROIDS;
    const uint8_t* cp = codes + int64_t(node) * code_stride;
    if constexpr (MS >= 8) {
      uint32_t w[MS / 4];
      if constexpr (MS == 8) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(cp));
        w[0] = v.x;
        w[1] = v.y;
      } else {
#pragma unroll
        for (int i = 0; i < MS / 16; ++i) {
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(cp) + i);
          w[4 * i + 0] = v.x;
          w[4 * i + 1] = v.y;
          w[4 * i + 2] = v.z;
          w[4 * i + 3] = v.w;
        }
      }
#pragma unroll
      for (int g = 0; g < QG; ++g) dist[g] = adc_sum_words<MS>(st + g * tsz, w);
    } else {
      uint8_t b[VECTRA_SCAN_MAX_SUBSPACES];
      for (int s = 0; s < m; ++s) b[s] = __ldg(cp + s);
#pragma unroll
      for (int g = 0; g < QG; ++g) dist[g] = adc_sum_bytes(st + g * tsz, b, m);
    }
  }
};

// ---------------------------------------------------------------------------
// Levels: score a sample (or every candidate), store or append keys.
// ---------------------------------------------------------------------------
struct Level {
  int64_t n_queries;
  int64_t n_rows;
  const int64_t* offsets;  // per-query candidates (CSR), or null: every row
  const uint32_t* ids;
  int64_t groups;          // sampled groups of 32 candidates; 0: every one
  int rows_per_lane;       // a CTA tile is 256 x rows_per_lane candidates
  int64_t n_slots;         // CTAs per query group
  const uint32_t* bound;   // admission keys; null: store every key (level 0)
  uint32_t* keys;          // [n_queries][cap]
  uint32_t* nodes;         // [n_queries][cap]
  uint32_t* count;         // [n_queries] entries stored or offered
  int64_t cap;
};

__device__ __forceinline__ int64_t cand_count(const Level& L, int64_t q) {
  return L.offsets == nullptr ? L.n_rows : L.offsets[q + 1] - L.offsets[q];
}

// One launch per level. A group's queries share their candidates (per-query
// candidate lists run with QG = 1). Scan index j of a query maps to its
// candidate j (every candidate) or to (j / 32) * spacing + j % 32 (a sample
// of groups of 32 consecutive candidates).
template <int QG, class Score>
__global__ void __launch_bounds__(kThreads)
    level_kernel(Score sc, Level L) {
  extern __shared__ __align__(16) float smem_f[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_groups = (L.n_queries + QG - 1) / QG;
  const int64_t group = blockIdx.x % n_groups;
  const int64_t slot = blockIdx.x / n_groups;
  const int64_t q0 = group * QG;
  const int64_t n = cand_count(L, q0);
  const bool every = L.groups == 0 || 32 * L.groups >= n;
  const int64_t m = every ? n : 32 * L.groups;
  const int64_t spacing = every ? 0 : n / L.groups;
  const int64_t tile = int64_t(kThreads) * L.rows_per_lane;
  const bool store_all = L.bound == nullptr;
  // Level 0 stores scan index j at entry j: no more than the buffer holds
  // (a query's list longer than the stated maximum is cut there).
  if (store_all && slot == 0 && threadIdx.x < QG &&
      q0 + threadIdx.x < L.n_queries)
    L.count[q0 + threadIdx.x] = uint32_t(m < L.cap ? m : L.cap);
  if (slot * tile >= m) return;
  sc.load(smem_f, q0, L.n_queries);
  __syncthreads();
  uint32_t bound[QG];
#pragma unroll
  for (int g = 0; g < QG; ++g)
    bound[g] = (!store_all && q0 + g < L.n_queries) ? L.bound[q0 + g]
                                                    : kNoBound;
  const int64_t id0 = L.offsets != nullptr ? L.offsets[q0] : 0;
  for (int64_t t = slot; t * tile < m; t += L.n_slots) {
    for (int r = 0; r < L.rows_per_lane; ++r) {
      const int64_t j0 = t * tile + (int64_t(r) * kWarps + warp) * 32;
      if (j0 >= m) break;  // warp-uniform
      const int64_t j = j0 + lane;
      const bool valid = j < m;
      const int64_t i = every ? j : (j >> 5) * spacing + (j & 31);
      const uint32_t node = !valid ? kNoNode
                            : L.offsets != nullptr ? L.ids[id0 + i]
                                                   : uint32_t(i);
      float dist[QG];
      if (valid) sc.score(smem_f, node, dist);
#pragma unroll
      for (int g = 0; g < QG; ++g) {
        const int64_t q = q0 + g;
        if (q >= L.n_queries) break;  // uniform
        const uint32_t key = valid ? dist_key(dist[g]) : kNoBound;
        uint32_t* qk = L.keys + q * L.cap;
        uint32_t* qn = L.nodes + q * L.cap;
        if (store_all) {
          if (valid && j < L.cap) {
            qk[j] = key;
            qn[j] = node;
          }
          continue;
        }
        const bool admit = valid && key <= bound[g];
        const unsigned bal = __ballot_sync(kFull, admit);
        if (bal == 0u) continue;
        const int leader = __ffs(bal) - 1;
        uint32_t pos = 0;
        if (lane == leader)
          pos = atomicAdd(L.count + q, uint32_t(__popc(bal)));
        pos = __shfl_sync(kFull, pos, leader) +
              uint32_t(__popc(bal & ((1u << lane) - 1u)));
        if (admit && pos < L.cap) {
          qk[pos] = key;
          qn[pos] = node;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// L2 levels over every row or a sample of groups of consecutive rows (no
// candidate lists), with dim = 64 * NC: rows reach shared memory by bulk
// copy and 16 lanes share a row.
//  * Each warp streams its own contiguous run of the CTA tile in batches of
//    8 consecutive rows (8 * row_stride floats), kBulkStages copies in
//    flight (one mbarrier each; waits bounded, timeouts set the device
//    error word).
//  * A step covers 4 rows of the batch: half-warp h takes rows 2 rho + h
//    (rho = 0, 1); lane l16 = lane % 16 holds floats [64 c + 4 l16, +4) of
//    chunk c of both rows and of each of the QG queries (in registers), so
//    it forms 2 QG partial sums.
//  * A butterfly over the 16 lanes adds them up: at each of the exchanges
//    (lane distance 8, 4, 2, 1) a lane keeps half of its values and adds its
//    partner's matching half, until one value is left. The lane's values
//    are laid out so that the half it keeps is always the first: item
//    (rho, g) sits at slot (rho, g) XOR F, F being the lane's final item,
//    by loading query g XOR F_g into query slot g and row rho XOR F_rho
//    into row slot rho. Every lane (every 2^k-th when 2 QG < 16) ends with
//    the distance of one (row, query) and stores or appends it.
// ---------------------------------------------------------------------------
constexpr int kBulkRows = 8;
constexpr int kBulkStages = 3;

struct L2Bulk {
  const float* queries;
  int64_t query_stride;
  const float* rows;
  int64_t row_stride;  // floats; a multiple of 4
  unsigned int* err;
};

template <int QG, int NC>
__global__ void __launch_bounds__(kThreads, 2)
    l2_bulk_kernel(L2Bulk b, Level L) {
  extern __shared__ __align__(128) unsigned char smem_b[];
  constexpr int V = 2 * QG;                        // values a lane starts with
  constexpr int kLogV = V >= 16 ? 4 : V == 8 ? 3 : V == 4 ? 2 : 1;
  constexpr int kDupShift = 4 - kLogV;             // lanes sharing a result
  constexpr int kLogQG = kLogV - 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_groups = (L.n_queries + QG - 1) / QG;
  const int64_t group = blockIdx.x % n_groups;
  const int64_t slot = blockIdx.x / n_groups;
  const int64_t q0 = group * QG;
  const int64_t n = L.n_rows;
  const bool every = L.groups == 0 || 32 * L.groups >= n;
  const int64_t m = every ? n : 32 * L.groups;
  const int64_t spacing = every ? 0 : n / L.groups;
  const int64_t tile = int64_t(kThreads) * L.rows_per_lane;
  const bool store_all = L.bound == nullptr;
  if (store_all && slot == 0 && threadIdx.x < QG &&
      q0 + threadIdx.x < L.n_queries)
    L.count[q0 + threadIdx.x] = uint32_t(m < L.cap ? m : L.cap);
  if (slot * tile >= m) return;

  const uint32_t stage_bytes =
      uint32_t(kBulkRows * b.row_stride * sizeof(float));
  float* wbuf = reinterpret_cast<float*>(smem_b) +
                size_t(warp) * kBulkStages * kBulkRows * b.row_stride;
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      smem_b + size_t(kWarps) * kBulkStages * stage_bytes);
  const uint32_t bar0 = smem_addr(bars + warp * kBulkStages);
  if (lane == 0) {
#pragma unroll
    for (int st = 0; st < kBulkStages; ++st) mbar_init(bar0 + 8 * st, 1);
    fence_barrier_init();
  }
  __syncwarp();

  // The lane's final item F = (rho_f, g_f) and its slot permutation.
  const int l16 = lane & 15, half = lane >> 4;
  const int f_item = l16 >> kDupShift;
  const int f_rho = f_item >> kLogQG, f_g = f_item & (QG - 1);
  const bool owner = (l16 & ((1 << kDupShift) - 1)) == 0 &&
                     q0 + f_g < L.n_queries;
  const int64_t my_q = q0 + f_g;
  const uint32_t my_bound =
      (!store_all && owner) ? L.bound[my_q] : kNoBound;
  // Query slot g holds query g ^ f_g: chunk c, lane slice l16, in pairs.
  uint64_t qp[QG][NC][2];
#pragma unroll
  for (int g = 0; g < QG; ++g) {
    const int64_t qq = q0 + (g ^ f_g);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (qq < L.n_queries) {
        const float* qs = b.queries + qq * b.query_stride + 64 * c + 4 * l16;
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = __ldg(qs + e);
      }
      qp[g][c][0] = pk(v[0], v[1]);
      qp[g][c][1] = pk(v[2], v[3]);
    }
  }

  // The warp's batches: in tile t, scan indices [t * tile + warp * run,
  // + run) in batches of 8; they stay below m for a prefix of the sequence.
  const int64_t run = tile / kWarps;
  const int64_t per_tile = run / kBulkRows;
  auto batch_j0 = [&](int64_t u) {
    const int64_t t = slot + (u / per_tile) * L.n_slots;
    return t * tile + warp * run + (u % per_tile) * kBulkRows;
  };
  const uint64_t policy = l2_evict_first_policy();
  auto issue = [&](int64_t u) {  // lane 0
    const int64_t j0 = batch_j0(u);
    const int64_t nv = m - j0 < kBulkRows ? m - j0 : kBulkRows;
    const int64_t i0 = every ? j0 : (j0 >> 5) * spacing + (j0 & 31);
    const int st = int(u % kBulkStages);
    // The batch's rows from the first one's start to the last one's final
    // element (64 * NC floats): a row view that ends where its storage ends
    // (a suffix of each row's columns) is never read past. Both terms are
    // multiples of 16 bytes, as the bulk copy requires.
    const uint32_t bytes =
        uint32_t(((nv - 1) * b.row_stride + 64 * NC) * sizeof(float));
    mbar_arrive_expect_tx(bar0 + 8 * st, bytes);
    bulk_g2s(smem_addr(wbuf + size_t(st) * kBulkRows * b.row_stride),
             b.rows + i0 * b.row_stride, bytes, bar0 + 8 * st, policy);
  };
  int64_t issued = 0;  // the same on every lane
  for (; issued < kBulkStages && batch_j0(issued) < m; ++issued)
    if (lane == 0) issue(issued);

  bool failed = false;
  int64_t u = 0;
  for (; batch_j0(u) < m; ++u) {
    const int st = int(u % kBulkStages);
    const uint32_t phase = uint32_t((u / kBulkStages) & 1);
    if (!mbar_wait(bar0 + 8 * st, phase, b.err)) {
      failed = true;
      ++u;
      break;
    }
    const int64_t j0 = batch_j0(u);
    const float* sb = wbuf + size_t(st) * kBulkRows * b.row_stride + 4 * l16;
#pragma unroll 1
    for (int step = 0; step < kBulkRows / 4; ++step) {
      float v[V];
#pragma unroll
      for (int rho = 0; rho < 2; ++rho) {
        // Row slot rho holds row 2 (rho ^ f_rho) + half of the step.
        const float* row = sb + (4 * step + 2 * (rho ^ f_rho) + half) *
                                    b.row_stride;
        uint64_t acc[QG];
#pragma unroll
        for (int g = 0; g < QG; ++g) acc[g] = 0;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const float4 rv = *reinterpret_cast<const float4*>(row + 64 * c);
          const uint64_t r01 = pk(rv.x, rv.y), r23 = pk(rv.z, rv.w);
#pragma unroll
          for (int g = 0; g < QG; ++g) {
            const uint64_t d01 = sub2(qp[g][c][0], r01);
            const uint64_t d23 = sub2(qp[g][c][1], r23);
            acc[g] = fma2(d01, d01, acc[g]);
            acc[g] = fma2(d23, d23, acc[g]);
          }
        }
#pragma unroll
        for (int g = 0; g < QG; ++g) {
          const float2 a2 = upk(acc[g]);
          v[rho * QG + g] = a2.x + a2.y;
        }
      }
      // The butterfly: keep the first half, add the partner's second.
      int cnt = V;
#pragma unroll
      for (int mm = 8; mm >= 1; mm >>= 1) {
        const int h = cnt >= 2 ? cnt / 2 : 1;
#pragma unroll
        for (int i = 0; i < h; ++i)
          v[i] += __shfl_xor_sync(kFull, v[cnt >= 2 ? i + h : i], mm);
        cnt = h;
      }
      const int64_t j = j0 + 4 * step + 2 * f_rho + half;
      if (!owner || j >= m) continue;
      const uint32_t key = dist_key(v[0]);
      const uint32_t node =
          uint32_t(every ? j : (j >> 5) * spacing + (j & 31));
      uint32_t* qk = L.keys + my_q * L.cap;
      uint32_t* qn = L.nodes + my_q * L.cap;
      if (store_all) {
        if (j < L.cap) {
          qk[j] = key;
          qn[j] = node;
        }
      } else if (key <= my_bound) {
        const uint32_t pos = atomicAdd(L.count + my_q, 1u);
        if (pos < L.cap) {
          qk[pos] = key;
          qn[pos] = node;
        }
      }
    }
    __syncwarp();  // every lane is done with the stage
    if (batch_j0(issued) < m) {  // refill it
      if (lane == 0) {
        fence_proxy_async_smem();
        issue(issued);
      }
      ++issued;
    }
  }
  if (failed) {  // let the copies still in flight land before returning
    for (; u < issued; ++u)
      mbar_wait(bar0 + 8 * int(u % kBulkStages),
                uint32_t((u / kBulkStages) & 1), b.err);
  }
}

// ---------------------------------------------------------------------------
// Select: the k smallest (key, node) values of a query's buffer.
// ---------------------------------------------------------------------------
enum SelectMode { kFirstBound = 0, kLowerBound = 1, kFinal = 2 };

struct Select {
  int64_t cap;
  int k;
  int mode;
  const uint32_t* keys;
  const uint32_t* nodes;
  uint32_t* count;     // read, then reset for the next level
  uint32_t* bound;     // per-query admission key (bound modes)
  float* out_d;        // final: results
  uint32_t* out_n;
  int32_t* counts;     // may be null
  int32_t* overflow;   // final: 1 where the buffer overflowed
  float* fb_d;         // final: the bound as a distance, for the re-scan
  uint32_t* fb_n;
};

// Exclusive prefix sum over the block's 1,024 threads; *total gets the sum.
__device__ __forceinline__ uint32_t block_scan(uint32_t v, uint32_t* wtot,
                                               uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(kFull, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wtot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const uint32_t w = wtot[lane];
    uint32_t s = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(kFull, s, o);
      if (lane >= o) s += y;
    }
    wtot[lane] = s - w;
    if (lane == 31) wtot[32] = s;
  }
  __syncthreads();
  const uint32_t r = wtot[warp] + x - v;
  *total = wtot[32];
  __syncthreads();  // wtot may be reused
  return r;
}

// Bitonic sort, ascending, of 32 << LOG_PER values held by one warp in
// registers: element e = j * 32 + lane in v[j]. Strides under 32 pair lanes
// (shuffles), larger ones a lane's own registers.
template <int LOG_PER>
__device__ __forceinline__ void warp_bitonic(
    unsigned long long (&v)[1 << LOG_PER], int lane) {
  constexpr int PER = 1 << LOG_PER;
#pragma unroll
  for (int ls = 1; ls <= 5 + LOG_PER; ++ls) {
    const int size = 1 << ls;
#pragma unroll
    for (int lt = ls - 1; lt >= 0; --lt) {
      const int stride = 1 << lt;
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const bool up = ((j * 32 + lane) & size) == 0;
        if (stride >= 32) {
          const int js = stride >> 5;
          if (j & js) continue;
          const unsigned long long x = v[j], y = v[j | js];
          if ((x > y) == up) {
            v[j] = y;
            v[j | js] = x;
          }
        } else {
          const unsigned long long o = __shfl_xor_sync(kFull, v[j], stride);
          const bool keep_min = ((lane & stride) == 0) == up;
          const bool less = v[j] < o;
          v[j] = keep_min ? (less ? v[j] : o) : (less ? o : v[j]);
        }
      }
    }
  }
}

// Bitonic sort, ascending, of p2 (a power of two) values in shared memory
// by threads t = 0 .. nt - 1: one warp (WARP, __syncwarp between stages) or
// the whole block (__syncthreads).
template <bool WARP>
__device__ __forceinline__ void smem_bitonic(unsigned long long* v,
                                             uint32_t p2, uint32_t t,
                                             uint32_t nt) {
#pragma unroll 1
  for (uint32_t size = 2; size <= p2; size <<= 1) {
#pragma unroll 1
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll 1
      for (uint32_t i = t; i < p2 / 2; i += nt) {
        const uint32_t lo = 2 * i - (i & (stride - 1));  // stride: 2^m
        const uint32_t hi = lo + stride;
        const bool up = (lo & size) == 0;
        const unsigned long long x = v[lo], y = v[hi];
        if ((x > y) == up) {
          v[lo] = y;
          v[hi] = x;
        }
      }
      if (WARP) {
        __syncwarp();
      } else {
        __syncthreads();
      }
    }
  }
}

// The bin of 2 * tid or 2 * tid + 1 holding rank r (from 1) of a histogram
// (2,048 bins, two per thread): pick = (bin, entries before it, in it).
__device__ __forceinline__ void pick_bin(const uint32_t* hist, uint32_t r,
                                         uint32_t* wtot, uint32_t* pick) {
  const int tid = threadIdx.x;
  const uint32_t h0 = hist[2 * tid], h1 = hist[2 * tid + 1];
  uint32_t total;
  const uint32_t ex = block_scan(h0 + h1, wtot, &total);
  if (ex < r && r <= ex + h0) {
    pick[0] = 2 * tid;
    pick[1] = ex;
    pick[2] = h0;
  } else if (ex + h0 < r && r <= ex + h0 + h1) {
    pick[0] = 2 * tid + 1;
    pick[1] = ex + h0;
    pick[2] = h1;
  }
}

// One CTA per query. The buffer's keys are staged in shared memory; loops
// stay rolled (each launch runs its code once, so a short kernel starts
// sooner).
__global__ void __launch_bounds__(kSelThreads) select_kernel(Select a) {
  extern __shared__ uint32_t skey[];  // [cap]
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t wtot[33];
  __shared__ uint32_t pick[3];
  __shared__ uint32_t span[64];
  __shared__ uint32_t n_sel_sh;
  __shared__ unsigned long long sorted[kSortMax];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t q = blockIdx.x;
  const uint32_t n_total = a.count[q];
  const int64_t n = int64_t(n_total) < a.cap ? int64_t(n_total) : a.cap;
  const uint32_t* qk = a.keys + q * a.cap;
  const uint32_t* qn = a.nodes + q * a.cap;
  uint32_t lo = kNoBound, hi = 0u;  // the keys' range, kept while staging
#pragma unroll 16
  for (int64_t i = tid; i < n; i += kSelThreads) {
    const uint32_t kv = qk[i];
    skey[i] = kv;
    lo = umin(lo, kv);
    hi = umax(hi, kv);
  }
  hist[tid] = 0u;
  hist[tid + kSelThreads] = 0u;
  if (tid == 0) n_sel_sh = 0u;
  __syncthreads();  // every thread has read the count
  if (tid == 0) a.count[q] = 0u;  // the next level appends from zero
  const uint32_t need = uint32_t(int64_t(a.k) < n ? int64_t(a.k) : n);
  if (a.mode == kFinal) {
    const bool over = n_total > a.cap;
    if (tid == 0) {
      // The re-scan runs only where this is set; it takes no bound (its
      // distances may round differently from the levels').
      a.overflow[q] = over ? 1 : 0;
      a.fb_d[q] = over ? INFINITY : -INFINITY;
      a.fb_n[q] = kNoNode;
    }
    if (over) return;  // the warp-list re-scan writes this query
    if (need == 0u) {
      for (int j = tid; j < a.k; j += kSelThreads) {
        a.out_d[q * a.k + j] = INFINITY;
        a.out_n[q * a.k + j] = kNoNode;
      }
      if (tid == 0 && a.counts != nullptr) a.counts[q] = 0;
      return;
    }
  } else if (need < uint32_t(a.k)) {  // fewer than k: no bound from here
    if (tid == 0 && a.mode == kFirstBound) a.bound[q] = kNoBound;
    return;
  }

  // First one histogram of the keys' offsets from their smallest, in 2,048
  // bins spanning their range. A bound needs no more: the last key of the
  // bin holding the need-th has at least need keys at or under it. A result
  // gathers the entries before that bin's end when they fit the sort buffer
  // (ranged).
  bool ranged = false;
  uint64_t range_end = 0;  // ranged: the keys under it are gathered
  if (n > kSortMax || a.mode != kFinal) {
    lo = __reduce_min_sync(kFull, lo);
    hi = __reduce_max_sync(kFull, hi);
    if (lane == 0) {
      span[warp] = lo;
      span[32 + warp] = hi;
    }
    __syncthreads();
    lo = __reduce_min_sync(kFull, span[lane]);
    hi = __reduce_max_sync(kFull, span[32 + lane]);
    const uint32_t range = hi - lo;
    const int shift = range < 2048u ? 0 : 32 - __clz(range) - 11;
#pragma unroll 4
    for (int64_t i = tid; i < n; i += kSelThreads)
      atomicAdd(&hist[(skey[i] - lo) >> shift], 1u);
    __syncthreads();
    pick_bin(hist, need, wtot, pick);
    hist[2 * tid] = 0u;
    hist[2 * tid + 1] = 0u;
    __syncthreads();
    ranged = pick[1] + pick[2] <= uint32_t(kSortMax);
    range_end = uint64_t(lo) + (uint64_t(pick[0] + 1) << shift);
    if (a.mode != kFinal) {
      if (tid == 0) {
        const uint32_t b = range_end - 1 > uint64_t(kNoBound)
                               ? kNoBound
                               : uint32_t(range_end - 1);
        a.bound[q] = a.mode == kFirstBound ? b : umin(a.bound[q], b);
      }
      return;
    }
    __syncthreads();  // pick is rewritten below
  }

  // Otherwise a radix select of the need-th smallest (key << 32 | node):
  // 11/11/10-bit digits of the key, then of the node, until the entries at
  // or under the bucket fit the sort buffer.
  uint64_t pre = 0;      // the selected digits so far, in place
  int pbits = 0;         // how many top bits they fix
  uint32_t below = 0;    // entries under the bucket
  uint32_t in_bucket = uint32_t(n);
#pragma unroll 1
  for (int round = 0;
       !ranged && round < 6 && below + in_bucket > uint32_t(kSortMax);
       ++round) {
    const int w = round % 3 == 2 ? 10 : 11;
    const int shift = 64 - pbits - w;
    const uint32_t pk32 = uint32_t(pre >> 32);
#pragma unroll 1
    for (int64_t base = int64_t(warp) * 32; base < n; base += kSelThreads) {
      const int64_t idx = base + lane;  // the warp iterates together
      bool inb = idx < n;
      uint32_t bin = 0;
      if (inb) {
        const uint32_t kv = skey[idx];
        if (pbits < 32) {
          inb = pbits == 0 || (kv >> (32 - pbits)) == (pk32 >> (32 - pbits));
          bin = (kv >> (shift - 32)) & ((1u << w) - 1u);
        } else {
          inb = kv == pk32;
          if (inb) {
            const uint32_t nd = qn[idx];
            const int nb = pbits - 32;
            inb = nb == 0 || (nd >> (32 - nb)) == (uint32_t(pre) >> (32 - nb));
            bin = (nd >> shift) & ((1u << w) - 1u);
          }
        }
      }
      const unsigned act = __ballot_sync(kFull, inb);
      if (inb) {
        const unsigned peers = __match_any_sync(act, bin);
        if (lane == __ffs(peers) - 1)
          atomicAdd(&hist[bin], uint32_t(__popc(peers)));
      }
    }
    __syncthreads();
    pick_bin(hist, need - below, wtot, pick);
    hist[2 * tid] = 0u;
    hist[2 * tid + 1] = 0u;
    __syncthreads();
    pre |= uint64_t(pick[0]) << shift;
    pbits += w;
    below += pick[1];
    in_bucket = pick[2];
    __syncthreads();  // pick is rewritten next round
  }

  // Gather the entries at or under the bucket (strictly under it when they
  // are copies of one value beyond the buffer) and sort them.
  const bool copies = !ranged && below + in_bucket > uint32_t(kSortMax);
  const uint32_t pk32 = uint32_t(pre >> 32), pn32 = uint32_t(pre);
#pragma unroll 1
  for (int64_t base = int64_t(warp) * 32; base < n; base += kSelThreads) {
    const int64_t idx = base + lane;
    bool s = false;
    uint32_t kv = 0u, nd = 0u;
    if (idx < n) {
      kv = skey[idx];
      if (ranged) {
        s = uint64_t(kv) < range_end;
      } else if (pbits == 0) {
        s = true;
      } else if (pbits <= 32) {
        s = (kv >> (32 - pbits)) <= (pk32 >> (32 - pbits));
      } else if (kv != pk32) {
        s = kv < pk32;
      } else {
        nd = qn[idx];
        s = copies ? nd < pn32 : (nd >> (64 - pbits)) <= (pn32 >> (64 - pbits));
      }
    }
    const unsigned bal = __ballot_sync(kFull, s);
    if (bal == 0u) continue;
    const int leader = __ffs(bal) - 1;
    uint32_t pos = 0u;
    if (lane == leader) pos = atomicAdd(&n_sel_sh, uint32_t(__popc(bal)));
    pos = __shfl_sync(kFull, pos, leader) +
          uint32_t(__popc(bal & ((1u << lane) - 1u)));
    if (s && pos < uint32_t(kSortMax))
      sorted[pos] = (uint64_t(kv) << 32) | qn[idx];
  }
  __syncthreads();
  const uint32_t n_sel = n_sel_sh < uint32_t(kSortMax) ? n_sel_sh
                                                       : uint32_t(kSortMax);
  uint32_t p2 = 2;
  while (p2 < n_sel) p2 <<= 1;
  if (p2 <= 128u) {  // one warp sorts in registers
    if (warp == 0) {
      unsigned long long v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t e = uint32_t(j * 32 + lane);
        v[j] = e < n_sel ? sorted[e] : ~0ull;
      }
      warp_bitonic<2>(v, lane);
#pragma unroll
      for (int j = 0; j < 4; ++j) sorted[j * 32 + lane] = v[j];
    }
  } else if (p2 <= 256u) {  // one warp sorts in shared memory
    if (warp == 0) {
      for (uint32_t i = n_sel + lane; i < p2; i += 32) sorted[i] = ~0ull;
      __syncwarp();
      smem_bitonic<true>(sorted, p2, lane, 32);
    }
  } else {
    for (uint32_t i = n_sel + tid; i < p2; i += kSelThreads) sorted[i] = ~0ull;
    __syncthreads();
    smem_bitonic<false>(sorted, p2, tid, kSelThreads);
  }
  __syncthreads();
  if (a.mode != kFinal) {
    if (tid == 0) {
      const uint32_t kth =
          uint32_t((copies && need > below ? pre : sorted[need - 1]) >> 32);
      a.bound[q] = a.mode == kFirstBound ? kth : umin(a.bound[q], kth);
    }
    return;
  }
  for (uint32_t j = tid; j < uint32_t(a.k); j += kSelThreads) {
    float d = INFINITY;
    uint32_t nd = kNoNode;
    if (j < need) {
      const uint64_t c = copies && j >= below ? pre : sorted[j];
      d = key_dist(uint32_t(c >> 32));
      nd = uint32_t(c);
    }
    a.out_d[q * a.k + j] = d;
    a.out_n[q * a.k + j] = nd;
  }
  if (tid == 0 && a.counts != nullptr) a.counts[q] = int32_t(need);
}

// ---------------------------------------------------------------------------
// The warp-list scan: exact for any input; re-does the queries whose last
// level overflowed its buffer.
// ---------------------------------------------------------------------------
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

struct ListShape {
  int64_t n_queries;
  int64_t n_rows;
  int64_t n_tiles;         // tiles of the largest candidate set
  int64_t n_slots;         // CTAs (and partial lists) per query group
  const int64_t* offsets;  // per-query candidates (CSR), or null
  const uint32_t* ids;
  const float* bound_d;    // per-query admission bound
  const uint32_t* bound_n;
  const int32_t* only;     // queries to scan (nonzero), or null: all
  int k;
};

// Candidate i of query q: its node id, or kNoNode.
__device__ __forceinline__ uint32_t candidate(const ListShape& sh, int64_t q,
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
                                           int64_t q0, int64_t slot,
                                           const ListShape& sh, float* wd,
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
    if (q0 + g >= sh.n_queries) continue;
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

template <int KPW, int QG, class Score>
__global__ void __launch_bounds__(kThreads)
    list_scan_kernel(Score sc, float* wd, uint32_t* wn, ListShape sh) {
  extern __shared__ __align__(16) float smem_f[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_groups = (sh.n_queries + QG - 1) / QG;
  const int64_t group = blockIdx.x % n_groups;
  const int64_t slot = blockIdx.x / n_groups;
  const int64_t q0 = group * QG;
  if (sh.only != nullptr) {
    bool any = false;
#pragma unroll
    for (int g = 0; g < QG; ++g)
      any |= q0 + g < sh.n_queries && sh.only[q0 + g] != 0;
    if (!any) return;
  }
  float* sq = smem_f;
  sc.load(sq, q0, sh.n_queries);
  __syncthreads();
  // The merge area follows the queries' floats.
  float* sd = smem_f + sc.floats();
  uint32_t* sn = reinterpret_cast<uint32_t*>(sd + QG * kWarps * KPW * 32);

  WarpList<KPW> lists[QG];
  float bd[QG];
  uint32_t bn[QG];
#pragma unroll
  for (int g = 0; g < QG; ++g) {
    lists[g].clear();
    const int64_t q = q0 + g;
    bd[g] = q < sh.n_queries ? sh.bound_d[q] : INFINITY;
    bn[g] = q < sh.n_queries ? sh.bound_n[q] : kNoNode;
  }
  for (int64_t tile = slot; tile < sh.n_tiles; tile += sh.n_slots)
    for (int r = 0; r < kMaxRowsPerLane; ++r) {
      const int64_t i =
          tile * kListTile + (int64_t(r) * kWarps + warp) * 32 + lane;
      // Candidates of a group's queries coincide (per-query lists use
      // QG = 1).
      const uint32_t node = candidate(sh, q0, i);
      float dist[QG];
      if (node != kNoNode) {
        sc.score(sq, node, dist);
      } else {
#pragma unroll
        for (int g = 0; g < QG; ++g) dist[g] = INFINITY;
      }
#pragma unroll
      for (int g = 0; g < QG; ++g) {
        const bool admit = !closer(bd[g], bn[g], dist[g], node);
        lists[g].offer(admit ? dist[g] : INFINITY, admit ? node : kNoNode,
                       sh.k, lane);
      }
    }
  merge_tile<KPW, QG>(lists, sd, sn, q0, slot, sh, wd, wn);
}

// Merge of a query's partial lists: one CTA per query; warp w merges slots
// w, w + 8, ... (the next batch's loads issued before the current batch is
// offered); warp 0 merges the eight lists.
template <int KPW>
__global__ void __launch_bounds__(kThreads)
    merge_kernel(const float* wd, const uint32_t* wn, ListShape sh,
                 float* out_d, uint32_t* out_n, int32_t* counts) {
  __shared__ float md[kWarps * KPW * 32];
  __shared__ uint32_t mn[kWarps * KPW * 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t q = blockIdx.x;
  if (sh.only != nullptr && sh.only[q] == 0) return;
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
  for (int i = KP; i < kWarps * KP; i += 32)
    m.offer(md[i + lane], mn[i + lane], k, lane);
#pragma unroll
  for (int s = 0; s < KPW; ++s) {
    const int j = s * 32 + lane;
    if (j < k) {
      out_d[q * k + j] = m.d[s];
      out_n[q * k + j] = m.n[s];
    }
  }
  if (counts != nullptr) {
    const int64_t nc = sh.offsets == nullptr
                           ? sh.n_rows
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

// Partial lists per query group at most (the warp-list scan's CTAs).
constexpr int64_t kMaxSlots = 512;

int64_t list_tiles(int64_t n_cand) {
  return n_cand > 0 ? (n_cand + kListTile - 1) / kListTile : 1;
}

// The levels of a scan of up to n_cand candidates per query: groups of 32
// sampled per level (0 = every candidate; the last level is always that).
struct Plan {
  int n_levels = 0;
  int64_t groups[8] = {};
  int64_t cap = 0;        // buffer entries per query
  bool rescan = false;    // the last level can overflow (warp-list re-scan)
};

Plan plan_for(int64_t n_cand, int k) {
  Plan p;
  if (n_cand <= kCap) {  // one level stores every candidate
    p.cap = std::max<int64_t>(n_cand, 1);
    p.groups[p.n_levels++] = 0;
    return p;
  }
  p.cap = kCap;
  p.rescan = true;
  int64_t s = kSample0;
  p.groups[p.n_levels++] = s / 32;
  // A level's bound is about the (k / s) quantile: the next level admits
  // about k * (its size) / s candidates. Go to every candidate once that is
  // at most a quarter of the buffer; else sample just enough for that (at
  // most what keeps this level's admissions to an eighth of the buffer).
  while (p.n_levels < 6 && int64_t(k) * n_cand > (kCap / 4) * s) {
    const int64_t enough = (int64_t(k) * n_cand + kCap / 4 - 1) / (kCap / 4);
    const int64_t most = s * (kCap / 8) / k;
    const int64_t s2 = (std::min(enough, most) + 31) / 32 * 32;
    if (2 * s2 >= n_cand) break;
    p.groups[p.n_levels++] = s2 / 32;
    s = s2;
  }
  p.groups[p.n_levels++] = 0;
  return p;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace: keys and nodes [n_queries][cap], then count, bound, overflow,
// re-scan bound (distance, node) [n_queries], then (plans that can overflow)
// the warp-list scan's partial lists [n_queries][slots][32 KPW] of
// distances and of nodes. Every part is written by a call before it reads
// it; nothing needs clearing between calls.
struct Workspace {
  uint32_t* keys;
  uint32_t* nodes;
  uint32_t* count;
  uint32_t* bound;
  int32_t* overflow;
  float* fb_d;
  uint32_t* fb_n;
  float* wd;
  uint32_t* wn;
};

size_t list_bytes(int64_t n_queries, int64_t n_cand, int k) {
  const int64_t slots = std::min(list_tiles(n_cand), kMaxSlots);
  return align256(size_t(n_queries) * size_t(slots) * size_t(kpw_for(k)) *
                  32 * 4);
}

size_t workspace_for(int64_t n_queries, int64_t n_cand, int k) {
  const Plan p = plan_for(n_cand, k);
  const size_t q = size_t(n_queries);
  size_t bytes = 2 * align256(q * size_t(p.cap) * 4) + 5 * align256(q * 4);
  if (p.rescan) bytes += 2 * list_bytes(n_queries, n_cand, k);
  return bytes + 256;
}

Workspace carve(void* base_ptr, int64_t n_queries, int64_t n_cand, int k) {
  const Plan p = plan_for(n_cand, k);
  const size_t q = size_t(n_queries);
  char* b = reinterpret_cast<char*>(
      (reinterpret_cast<uintptr_t>(base_ptr) + 255) & ~uintptr_t(255));
  Workspace w;
  const size_t buf = align256(q * size_t(p.cap) * 4), small = align256(q * 4);
  w.keys = reinterpret_cast<uint32_t*>(b);
  w.nodes = reinterpret_cast<uint32_t*>(b + buf);
  b += 2 * buf;
  w.count = reinterpret_cast<uint32_t*>(b);
  w.bound = reinterpret_cast<uint32_t*>(b + small);
  w.overflow = reinterpret_cast<int32_t*>(b + 2 * small);
  w.fb_d = reinterpret_cast<float*>(b + 3 * small);
  w.fb_n = reinterpret_cast<uint32_t*>(b + 4 * small);
  b += 5 * small;
  w.wd = nullptr;
  w.wn = nullptr;
  if (p.rescan) {
    const size_t lb = list_bytes(n_queries, n_cand, k);
    w.wd = reinterpret_cast<float*>(b);
    w.wn = reinterpret_cast<uint32_t*>(b + lb);
  }
  return w;
}

// Sets a kernel's dynamic shared-memory limit once per (kernel, device) and
// returns how many of its CTAs fit an SM with `smem` bytes. (Instantiations
// that differ only in template values share a function pointer type, so the
// record is kept by address.)
struct KernelRecord {
  const void* kern;
  int dev;
  size_t smem;
  int blocks;
};

cudaError_t prepare_kernel(const void* kern, size_t smem, int threads,
                           int* blocks_per_sm) {
  static std::mutex mu;
  static std::vector<KernelRecord> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  bool attr = false;
  for (const auto& e : done) {
    if (e.kern == kern && e.dev == dev) {
      attr = true;
      if (e.smem == smem) {
        *blocks_per_sm = e.blocks;
        return cudaSuccess;
      }
    }
  }
  cudaError_t err = cudaSuccess;
  if (!attr) {
    // Up to 227 KB per block, static shared memory included.
    cudaFuncAttributes fa;
    if ((err = cudaFuncGetAttributes(&fa, kern)) != cudaSuccess) return err;
    err = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
        int(227 * 1024 - fa.sharedSizeBytes));
  }
  if (err != cudaSuccess) return err;
  int blocks = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kern, threads,
                                                      smem);
  if (err != cudaSuccess) return err;
  blocks = std::max(blocks, 1);
  done.push_back({kern, dev, smem, blocks});
  *blocks_per_sm = blocks;
  return cudaSuccess;
}

struct Common {
  int64_t n_queries;
  int64_t n_rows;
  int64_t n_cand;  // the largest candidate set
  vectra_scan_candidates cand;
  vectra_scan_results res;
  int k;
};

// The levels and selects of one scan, then the warp-list re-scan of the
// queries whose last level overflowed (its CTAs return at once otherwise).
// Level launches: the lane-per-row kernel (any scorer, candidate lists) ...
template <int QG, class Score>
struct LaneLevels {
  Score sc;
  size_t smem;
  cudaError_t prepare(int* per_sm) const {
    return prepare_kernel(
        reinterpret_cast<const void*>(level_kernel<QG, Score>), smem,
        kThreads, per_sm);
  }
  void launch(unsigned blocks, const Level& L, cudaStream_t stream) const {
    level_kernel<QG, Score><<<dim3(blocks), kThreads, smem, stream>>>(sc, L);
  }
};

// ... or the bulk-copy L2 kernel.
template <int QG, int NC>
struct BulkLevels {
  L2Bulk b;
  size_t smem;
  cudaError_t prepare(int* per_sm) const {
    return prepare_kernel(reinterpret_cast<const void*>(l2_bulk_kernel<QG, NC>),
                          smem, kThreads, per_sm);
  }
  void launch(unsigned blocks, const Level& L, cudaStream_t stream) const {
    l2_bulk_kernel<QG, NC><<<dim3(blocks), kThreads, smem, stream>>>(b, L);
  }
};

template <int QG, class Score, class Levels>
cudaError_t run_levels(const Score& sc, size_t smem_floats,
                       const Levels& levels, const Common& c,
                       const Workspace& w, cudaStream_t stream) {
  const Plan p = plan_for(c.n_cand, c.k);
  const size_t smem = smem_floats * 4;  // the scorer's (re-scan kernel)
  int per_sm = 1;
  cudaError_t err = levels.prepare(&per_sm);
  if (err != cudaSuccess) return err;
  const size_t sel_smem = size_t(p.cap) * 4;
  int sel_per_sm = 1;
  err = prepare_kernel(reinterpret_cast<const void*>(select_kernel), sel_smem,
                       kSelThreads, &sel_per_sm);
  if (err != cudaSuccess) return err;
  const int64_t n_groups = (c.n_queries + QG - 1) / QG;
  const int64_t target = std::max<int64_t>(
      1, (int64_t(per_sm) * device_sm_count() + n_groups - 1) / n_groups);
  for (int l = 0; l < p.n_levels; ++l) {
    Level L;
    L.n_queries = c.n_queries;
    L.n_rows = c.n_rows;
    L.offsets = c.cand.offsets;
    L.ids = c.cand.ids;
    L.groups = p.groups[l];
    const int64_t m = (L.groups == 0 || 32 * L.groups >= c.n_cand)
                          ? c.n_cand
                          : 32 * L.groups;
    const int64_t tiles1 =
        std::max<int64_t>(1, (m + kThreads - 1) / kThreads);
    L.rows_per_lane = int(std::min<int64_t>(
        kMaxRowsPerLane,
        std::max<int64_t>(1, (tiles1 + target - 1) / target)));
    const int64_t tile = int64_t(kThreads) * L.rows_per_lane;
    L.n_slots = std::max<int64_t>(1, std::min(target, (m + tile - 1) / tile));
    L.bound = l == 0 ? nullptr : w.bound;
    L.keys = w.keys;
    L.nodes = w.nodes;
    L.count = w.count;
    L.cap = p.cap;
    const int64_t blocks = n_groups * L.n_slots;
    if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
    levels.launch(unsigned(blocks), L, stream);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    Select s;
    s.cap = p.cap;
    s.k = c.k;
    s.mode = l + 1 == p.n_levels ? kFinal : l == 0 ? kFirstBound : kLowerBound;
    s.keys = w.keys;
    s.nodes = w.nodes;
    s.count = w.count;
    s.bound = w.bound;
    s.out_d = c.res.distances;
    s.out_n = c.res.nodes;
    s.counts = c.res.counts;
    s.overflow = w.overflow;
    s.fb_d = w.fb_d;
    s.fb_n = w.fb_n;
    select_kernel<<<dim3(unsigned(c.n_queries)), kSelThreads, sel_smem,
                    stream>>>(s);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  }
  if (!p.rescan) return cudaSuccess;
  // The warp-list re-scan.
  auto go = [&](auto kpw_tag) -> cudaError_t {
    constexpr int KPW = decltype(kpw_tag)::value;
    const size_t lsmem = smem + size_t(QG) * kWarps * KPW * 32 * 8;
    if (lsmem > 227 * 1024) return cudaErrorInvalidConfiguration;
    int lper = 1;
    cudaError_t e = prepare_kernel(
        reinterpret_cast<const void*>(list_scan_kernel<KPW, QG, Score>),
        lsmem, kThreads, &lper);
    if (e != cudaSuccess) return e;
    ListShape sh;
    sh.n_queries = c.n_queries;
    sh.n_rows = c.n_rows;
    sh.n_tiles = list_tiles(c.n_cand);
    sh.n_slots = std::max<int64_t>(
        1, std::min({(int64_t(2) * device_sm_count() + n_groups - 1) /
                         n_groups,
                     sh.n_tiles, kMaxSlots}));
    sh.offsets = c.cand.offsets;
    sh.ids = c.cand.ids;
    sh.bound_d = w.fb_d;
    sh.bound_n = w.fb_n;
    sh.only = w.overflow;
    sh.k = c.k;
    const int64_t blocks = n_groups * sh.n_slots;
    list_scan_kernel<KPW, QG, Score>
        <<<dim3(unsigned(blocks)), kThreads, lsmem, stream>>>(sc, w.wd, w.wn,
                                                              sh);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    merge_kernel<KPW><<<dim3(unsigned(c.n_queries)), kThreads, 0, stream>>>(
        w.wd, w.wn, sh, c.res.distances, c.res.nodes, c.res.counts);
    return cudaGetLastError();
  };
  switch (kpw_for(c.k)) {
    case 1: return go(std::integral_constant<int, 1>());
    case 2: return go(std::integral_constant<int, 2>());
    case 4: return go(std::integral_constant<int, 4>());
    default: return go(std::integral_constant<int, 8>());
  }
}

// Queries per CTA: up to 8, no more than needed for the queries, with their
// vectors or tables and the re-scan's merge area within 200 KB of shared
// memory, for scans of every row; 1 for per-query candidate lists.
int group_for(int64_t n_queries, bool shared_candidates,
              size_t per_query_bytes, int k) {
  if (!shared_candidates) return 1;
  const size_t lists = size_t(kWarps) * kpw_for(k) * 32 * 8;
  int qg = 8;
  while (qg > 1 && (qg / 2 >= n_queries ||
                    size_t(qg) * (per_query_bytes + lists) >
                        size_t(200) * 1024))
    qg /= 2;
  return qg;
}

template <template <int> class Run, typename... A>
cudaError_t by_group(int qg, A... args) {
  switch (qg) {
    case 8: return Run<8>::go(args...);
    case 4: return Run<4>::go(args...);
    case 2: return Run<2>::go(args...);
    default: return Run<1>::go(args...);
  }
}

template <int QG>
struct L2Run {
  static cudaError_t go(const vectra_scan_l2_args* a, const Common* c,
                        const Workspace* w, cudaStream_t stream) {
    L2Score<QG> sc;
    sc.queries = a->queries;
    sc.query_stride = a->query_stride;
    sc.rows = a->rows;
    sc.row_stride = a->row_stride;
    sc.dim = a->dimension;
    sc.vec4 = (a->dimension % 4 == 0) && (a->row_stride % 4 == 0) &&
              (reinterpret_cast<uintptr_t>(a->rows) % 16 == 0);
    const size_t sf = L2Score<QG>::smem_floats(a->dimension);
    // Rows of every candidate (no lists), 16-byte aligned, dim = 64 NC with
    // the queries' slices fitting 64 registers: the bulk-copy kernel.
    const int nc = a->dimension / 64;
    const bool bulk = c->cand.offsets == nullptr && sc.vec4 &&
                      a->dimension % 64 == 0 && a->row_stride <= 256 &&
                      (nc == 1 || nc == 2 || nc == 4) && QG * nc <= 16;
    if (bulk) {
      L2Bulk b{a->queries, a->query_stride, a->rows, a->row_stride,
               device_error_ptr()};
      const size_t smem = size_t(kWarps) * kBulkStages * kBulkRows *
                              a->row_stride * sizeof(float) +
                          size_t(kWarps) * kBulkStages * 8;
      if constexpr (QG <= 4) {
        if (nc == 4)
          return run_levels<QG>(sc, sf, BulkLevels<QG, 4>{b, smem}, *c, *w,
                                stream);
      }
      if constexpr (QG <= 8) {
        if (nc == 2)
          return run_levels<QG>(sc, sf, BulkLevels<QG, 2>{b, smem}, *c, *w,
                                stream);
      }
      return run_levels<QG>(sc, sf, BulkLevels<QG, 1>{b, smem}, *c, *w,
                            stream);
    }
    return run_levels<QG>(sc, sf, LaneLevels<QG, L2Score<QG>>{sc, sf * 4}, *c,
                          *w, stream);
  }
};

template <int QG>
struct PqRun {
  template <int MS>
  static cudaError_t with(const vectra_scan_pq_args* a, const Common* c,
                          const Workspace* w, cudaStream_t stream) {
    PqScore<QG, MS> sc;
    sc.tables = a->tables;
    sc.codes = a->codes;
    sc.code_stride = a->code_stride;
    sc.m = a->subspaces;
    const size_t sf = PqScore<QG, MS>::smem_floats(a->subspaces);
    return run_levels<QG>(sc, sf, LaneLevels<QG, PqScore<QG, MS>>{sc, sf * 4},
                          *c, *w, stream);
  }
  static cudaError_t go(const vectra_scan_pq_args* a, const Common* c,
                        const Workspace* w, cudaStream_t stream) {
    const uintptr_t base = reinterpret_cast<uintptr_t>(a->codes);
    const bool a16 = base % 16 == 0 && a->code_stride % 16 == 0;
    const bool a8 = base % 8 == 0 && a->code_stride % 8 == 0;
    switch (a->subspaces) {
      case 8: return a8 ? with<8>(a, c, w, stream) : with<0>(a, c, w, stream);
      case 16:
        return a16 ? with<16>(a, c, w, stream) : with<0>(a, c, w, stream);
      case 32:
        return a16 ? with<32>(a, c, w, stream) : with<0>(a, c, w, stream);
      case 64:
        return a16 ? with<64>(a, c, w, stream) : with<0>(a, c, w, stream);
      default: return with<0>(a, c, w, stream);
    }
  }
};

// Common argument checks; the workspace carved.
int prepare(int64_t n_queries, int64_t n_rows, int k,
            const vectra_scan_candidates& cand,
            const vectra_scan_results& res, void* workspace,
            size_t workspace_bytes, Common* c, Workspace* w) {
  if (res.distances == nullptr || res.nodes == nullptr) return VECTRA_ERR_NULL;
  if (n_queries < 0 || n_rows < 0 || n_rows >= 0xffffffffLL ||
      n_queries > 0x7fffffffLL)
    return VECTRA_ERR_SHAPE;
  if (k < 1 || k > VECTRA_SCAN_MAX_K) return VECTRA_ERR_UNSUPPORTED;
  if (cand.offsets != nullptr &&
      (cand.ids == nullptr || cand.max_per_query < 0 ||
       cand.max_per_query >= 0xffffffffLL))
    return VECTRA_ERR_NULL;
  const int64_t nc = cand.offsets == nullptr ? n_rows : cand.max_per_query;
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 15) ||
      workspace_bytes < workspace_for(n_queries, nc, k))
    return VECTRA_ERR_NULL;
  c->n_queries = n_queries;
  c->n_rows = n_rows;
  c->n_cand = nc;
  c->cand = cand;
  c->res = res;
  c->k = k;
  *w = carve(workspace, n_queries, nc, k);
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
  Common c;
  Workspace w;
  const int st = prepare(a->n_queries, a->n_rows, a->k, a->candidates,
                         a->results, a->workspace, a->workspace_bytes, &c,
                         &w);
  if (st != VECTRA_OK) return st;
  if (a->n_queries == 0) return VECTRA_OK;
  const int qg = group_for(a->n_queries, a->candidates.offsets == nullptr,
                           size_t((a->dimension + 3) & ~3) * 4, a->k);
  return by_group<L2Run>(qg, a, &c, &w, s) == cudaSuccess ? VECTRA_OK
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
  Common c;
  Workspace w;
  const int st = prepare(a->n_queries, a->n_rows, a->k, a->candidates,
                         a->results, a->workspace, a->workspace_bytes, &c,
                         &w);
  if (st != VECTRA_OK) return st;
  if (a->n_queries == 0) return VECTRA_OK;
  const int qg = group_for(a->n_queries, a->candidates.offsets == nullptr,
                           size_t(a->subspaces) * VECTRA_PQ_CENTROIDS * 4,
                           a->k);
  return by_group<PqRun>(qg, a, &c, &w, s) == cudaSuccess ? VECTRA_OK
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
