// rbf_small.cu: RBF attention for planes whose keys fit one tile
// (1 <= Nk <= 128), any Nq >= 2, bf16/f16, D == Dv in {32, 64}. This is the
// compiled price model's attention site (benchmark config 5: per site
// B=1024, H=8, Nq=Nk=65, D=32, q/k/v strided views of one projection,
// models/price_transformer/spatial_attention.py:68-88).
//
// Design (B200):
//  * Work item: (plane, block of QR = 16 W queries); the CTA has W warps
//    (W = ceil(min(Nq, 128) / 16)) and warp w owns queries 16w..16w+15 of
//    the block. Persistent CTAs, several per SM, walk their items through a
//    ring of kStages stages. A stage holds the item's Q block and the
//    plane's K and V, each one TMA box of a 4-D tensor map over the
//    caller's strides (rows past Nq / Nk arrive as zeros; no host copy of
//    the strided views), swizzled over the row (64 B for D = 32, 128 B for
//    D = 64) so the ldmatrix reads below are free of bank conflicts.
//  * Every warp consumes every item, in order, so a parity wait on the
//    stage's mbarrier is exact. The last warp done with an item (counted
//    with an acq_rel shared-memory atomic) refills the stage with the item
//    kStages ahead.
//  * Logits are 2 g q.k_j - g ||k_j||^2 + b_j in the exp2 domain (the
//    row-constant -g ||q||^2 cancels in the softmax). The key terms
//    (b_j - g ||k_j||^2) log2(e) are formed once per item from the staged
//    K by every thread of the CTA (two adjacent lanes per key when the CTA
//    has two threads per key, each taking half of the key's chunks, joined
//    by one shuffle), so no warp waits long at the barrier that publishes
//    them; the scale and bias loads are issued before the stage wait so
//    their latency overlaps it.
//  * Item coordinates (b, h, query block) advance by a fixed step per item
//    (no integer division in the loop); the row sums use packed f32x2
//    adds; when the key tile's last 8 keys are all padding (Nk <= NKP - 8,
//    e.g. 65 keys in an 80-key tile) that n-tile of S is not computed and
//    its P is zero.
//  * S = Q K^T and O = P V on mma.sync m16n8k16 (bf16/f16 in, f32
//    accumulate): Q fragments by ldmatrix, K fragments by ldmatrix, V
//    fragments by ldmatrix.trans. All of a plane's keys are in the tile, so
//    the softmax is exact in one pass: row max and sum over the four lanes
//    that share a row, the reference's safe-max rule for rows with every
//    key masked (kernels/vectra_kernels/reference.py:146-152; they end as
//    0/0 = NaN), and P rounded to the input type before P V, as the
//    reference kernel does (spatial_rbf_attention.py:158-165). P is reused
//    from the S accumulators as A fragments (no shared-memory round trip).
#include <atomic>

#include "mma_sync.cuh"
#include "rbf_common.cuh"

namespace vectra {
namespace {

// Stages of the ring (each one item: Q block, K and V of a plane). Two
// measured best on the config-5 site (51.4 us; 3 stages 52.0 us, 4 stages
// 61.4 us): fewer bytes per CTA leave room for more CTAs per SM.
#ifndef VECTRA_SMALL_STAGES
#define VECTRA_SMALL_STAGES 2
#endif
constexpr int kStages = VECTRA_SMALL_STAGES;
// 1: an 8-key tile of S whose keys are all padding (Nk <= NKP - 8) is not
// computed.
#ifndef VECTRA_SMALL_TRIM_KEYS
#define VECTRA_SMALL_TRIM_KEYS 1
#endif
// 1: two threads per key form the key terms when the CTA has 2 NKP threads.
#ifndef VECTRA_SMALL_SPLIT_KEYS
#define VECTRA_SMALL_SPLIT_KEYS 1
#endif

struct SmallLaunch {
  int qr;           // queries per item (16 W)
  int nqb;          // query blocks per plane
  int n_items;      // B * H * nqb
  int H;
  int stage_bytes;  // one stage: Q block | K | V, each 1024-byte aligned
  int k_off;
  int v_off;
};

__host__ __device__ constexpr int align1k(int x) { return (x + 1023) & ~1023; }

// Byte offset of 16-byte chunk `chunk` of row `row` in a TMA tile whose rows
// are RB bytes, swizzled over the row (SWIZZLE_128B / SWIZZLE_64B: address
// bits [7, 7+log2(RB/16)) are XORed into the chunk index bits [4, ...)).
template <int RB>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  static_assert(RB == 64 || RB == 128, "row bytes");
  const int x = RB == 128 ? (row & 7) : ((row >> 1) & 3);
  return uint32_t(row * RB + ((chunk ^ x) << 4));
}

__device__ __forceinline__ uint32_t atomic_add_acq_rel(uint32_t addr,
                                                       uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "r"(addr), "r"(v)
               : "memory");
  return old;
}

// Packed float32 pairs (sm_100a f32x2 arithmetic) for the softmax's row
// sums.
__device__ __forceinline__ uint64_t f2pk(float x, float y) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
  return r;
}
__device__ __forceinline__ float2 f2upk(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// (b, h, query block) of a CTA's items, walked without divisions: item i of
// the CTA is global item blockIdx.x + i * gridDim.x, and consecutive items
// differ by gridDim.x = (db planes of H, dh heads, dq query blocks).
struct ItemCursor {
  int b, h, qb;
  __device__ void init(int item, const SmallLaunch& L) {
    const int plane = item / L.nqb;
    qb = item - plane * L.nqb;
    b = plane / L.H;
    h = plane - b * L.H;
  }
  __device__ void advance(int dq, int dh, int db, const SmallLaunch& L) {
    qb += dq;
    int carry = 0;
    if (qb >= L.nqb) {
      qb -= L.nqb;
      carry = 1;
    }
    h += dh + carry;
    if (h >= L.H) {
      h -= L.H;
      b += 1;
    }
    b += db;
  }
};

// PARTS threads (adjacent lanes) share a key's norm: each takes CH / PARTS
// of its 16-byte chunks and they add their partial sums with a shuffle, so
// the key terms are spread over every thread of the CTA.
template <typename T, int D, int NKP, int PARTS, int NTV>
__global__ void __launch_bounds__(256)
    rbf_small_kernel(const __grid_constant__ CUtensorMap tq,
                     const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, RbfProblem p,
                     SmallLaunch L) {
  static_assert(D == 32 || D == 64, "head width");
  static_assert(NKP % 16 == 0 && NKP <= 128, "key tile");
  constexpr int RB = D * 2;        // bytes per row (bf16/f16)
  constexpr int CH = RB / 16;      // 16-byte chunks per row
  constexpr int NT = NKP / 8;      // 8-key n-tiles of S
  static_assert(NTV >= NT - 1 && NTV <= NT, "valid n-tiles");
  constexpr int KS = D / 16;       // 16-dim k-steps of S
  constexpr int DT = D / 8;        // 8-dim n-tiles of O
  // Key-term slots per thread: with two threads per key the CTA has at
  // least 2 NKP threads, so one slot covers the tile.
  constexpr int BPT = PARTS == 2 ? 1 : 4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  float* terms = reinterpret_cast<float*>(smem + kStages * L.stage_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(terms + kStages * NKP);
  uint32_t* count = reinterpret_cast<uint32_t*>(full + kStages);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int W = blockDim.x >> 5, nthreads = blockDim.x;
  const int g = lane >> 2, c = lane & 3;
  const int nk = static_cast<int>(p.Nk);
  const int nq = static_cast<int>(p.Nq);
  const uint32_t tx_bytes = uint32_t(L.qr * RB + 2 * NKP * RB);
  static_assert(PARTS == 1 || PARTS == 2, "key-term split");
  static_assert(CH % PARTS == 0, "chunks per part");
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      count[s] = 0;
    }
    fence_barrier_init();
  }
  allow_dependents();
  __syncthreads();
  grid_dependency_wait();  // before any global access

  // Item i of this CTA is global item blockIdx.x + i * gridDim.x.
  const int my_items =
      L.n_items > int(blockIdx.x)
          ? (L.n_items - 1 - int(blockIdx.x)) / int(gridDim.x) + 1
          : 0;
  const int gstep = int(gridDim.x);
  const int dq = gstep % L.nqb, dplanes = gstep / L.nqb;
  const int dh = dplanes % L.H, db = dplanes / L.H;
  auto issue = [&](int i, const ItemCursor& cur) {  // one thread
    const int s = i % kStages;
    uint8_t* st = stages + size_t(s) * L.stage_bytes;
    const uint32_t bar = smem_addr(&full[s]);
    mbar_arrive_expect_tx(bar, tx_bytes);
    tma_load_4d(smem_addr(st), &tq, bar, 0, cur.qb * L.qr, cur.h, cur.b);
    tma_load_4d(smem_addr(st + L.k_off), &tk, bar, 0, 0, cur.h, cur.b);
    tma_load_4d(smem_addr(st + L.v_off), &tv, bar, 0, 0, cur.h, cur.b);
  };
  // Every thread walks `cur` (item i) without divisions; the thread that
  // refills a stage places its item (i + kStages) from scratch.
  ItemCursor cur;
  cur.init(int(blockIdx.x), L);
  if (tid == 0)
    for (int i = 0; i < kStages && i < my_items; ++i) {
      ItemCursor at;
      at.init(int(blockIdx.x) + i * gstep, L);
      issue(i, at);
    }

  for (int i = 0; i < my_items; ++i) {
    const int b = cur.b, h = cur.h, qb = cur.qb;
    cur.advance(dq, dh, db, L);
    const int s = i % kStages;
    uint8_t* st = stages + size_t(s) * L.stage_bytes;
    float* term = terms + s * NKP;

    // Scale and the key biases this thread finalises (its keys u / PARTS,
    // u = tid + t * nthreads, where u % PARTS == 0), loaded before the stage
    // wait so their latency overlaps it. (Loading them a whole item ahead
    // measured slower: the registers they hold cost more than they hide.)
    const float gamma = load_scale(p, b, h);
    float bias[BPT];
#pragma unroll
    for (int t = 0; t < BPT; ++t) {
      const int u = tid + t * nthreads;
      const int j = u / PARTS;
      bias[t] = 0.f;
      if (u % PARTS == 0 && j < nk && p.bias != nullptr)
        bias[t] = load_bias(p, b, h, j);
    }

    const bool ok = mbar_wait_sleep(smem_addr(&full[s]),
                                    uint32_t((i / kStages) & 1), p.err);
    if (ok) {
      // Key terms (b_j - g ||k_j||^2) log2(e); -inf for padded keys.
#pragma unroll
      for (int t = 0; t < BPT; ++t) {
        const int u = tid + t * nthreads;
        if (u - lane >= NKP * PARTS) break;  // warp-uniform
        const int j = u / PARTS, part = u % PARTS;
        float acc = 0.f;
        if (j < nk) {
#pragma unroll
          for (int cc = 0; cc < CH / PARTS; ++cc) {
            const uint4 raw = *reinterpret_cast<const uint4*>(
                st + L.k_off + swz<RB>(j, part + cc * PARTS));
            const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
            for (int x = 0; x < 8; ++x) {
              const float f = to_f32(e[x]);
              acc = fmaf(f, f, acc);
            }
          }
        }
        if (PARTS == 2) acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        if (part == 0 && j < NKP) {
          float v = kNegInf;
          if (j < nk && bias[t] != kNegInf)
            v = (bias[t] - gamma * acc) * kLog2e;
          term[j] = v;
        }
      }
    }
    if (__syncthreads_or(!ok)) return;  // error recorded; all threads leave

    const int q0 = qb * L.qr + warp * 16;  // this warp's first query
    if (q0 < nq) {
      const uint32_t qbase = smem_addr(st), kbase = smem_addr(st + L.k_off);
      const uint32_t vbase = smem_addr(st + L.v_off);
      // Q fragments (rows 16 warp .. +15 of the block).
      uint32_t qa[KS][4];
#pragma unroll
      for (int ks = 0; ks < KS; ++ks)
        ldsm_x4(qbase + swz<RB>(warp * 16 + (lane & 15), 2 * ks + (lane >> 4)),
                qa[ks]);
      // S = Q K^T.
      float sc[NT][4];
#pragma unroll
      for (int j = 0; j < NT; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t kb[4];
          ldsm_x4(kbase + swz<RB>(16 * np + (lane & 7) + ((lane >> 4) << 3),
                                  2 * ks + ((lane >> 3) & 1)),
                  kb);
          mma16816<T>(sc[2 * np], qa[ks], kb[0], kb[1]);
          if (2 * np + 1 < NTV)
            mma16816<T>(sc[2 * np + 1], qa[ks], kb[2], kb[3]);
        }
      }
      // Logits, exact row softmax over the quad sharing a row.
      const float g2 = 2.f * gamma * kLog2e;
      float m0 = kNegInf, m1 = kNegInf;
#pragma unroll
      for (int j = 0; j < NTV; ++j) {
        const float2 t2 = *reinterpret_cast<const float2*>(&term[8 * j + 2 * c]);
        sc[j][0] = fmaf(sc[j][0], g2, t2.x);
        sc[j][1] = fmaf(sc[j][1], g2, t2.y);
        sc[j][2] = fmaf(sc[j][2], g2, t2.x);
        sc[j][3] = fmaf(sc[j][3], g2, t2.y);
        m0 = fmax3(m0, sc[j][0], sc[j][1]);
        m1 = fmax3(m1, sc[j][2], sc[j][3]);
      }
      m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 1));
      m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
      m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
      m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
      const float s0 = m0 == kNegInf ? 0.f : m0;
      const float s1 = m1 == kNegInf ? 0.f : m1;
      uint64_t l0x2 = 0, l1x2 = 0;
      uint32_t pa[NT][2];  // P as packed pairs: [tile][row g, row g + 8]
#pragma unroll
      for (int j = 0; j < NTV; ++j) {
        const float p0 = fast_exp2(sc[j][0] - s0), p1 = fast_exp2(sc[j][1] - s0);
        const float p2 = fast_exp2(sc[j][2] - s1), p3 = fast_exp2(sc[j][3] - s1);
        l0x2 = fadd2(l0x2, f2pk(p0, p1));
        l1x2 = fadd2(l1x2, f2pk(p2, p3));
        pa[j][0] = pack_pair<T>(p0, p1);
        pa[j][1] = pack_pair<T>(p2, p3);
      }
#pragma unroll
      for (int j = NTV; j < NT; ++j) pa[j][0] = pa[j][1] = 0u;  // padding
      const float2 l0p = f2upk(l0x2), l1p = f2upk(l1x2);
      float l0 = l0p.x + l0p.y, l1 = l1p.x + l1p.y;
      l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
      l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
      // O = P V. (Separate accumulators for even and odd 16-key steps, to
      // shorten the dependency chains, measured slower.)
      float o[DT][4];
#pragma unroll
      for (int j = 0; j < DT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < NKP / 16; ++kk) {
        const uint32_t a[4] = {pa[2 * kk][0], pa[2 * kk][1], pa[2 * kk + 1][0],
                               pa[2 * kk + 1][1]};
#pragma unroll
        for (int dp = 0; dp < D / 16; ++dp) {
          uint32_t vb[4];
          ldsm_x4_t(vbase + swz<RB>(16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3),
                                    2 * dp + (lane >> 4)),
                    vb);
          mma16816<T>(o[2 * dp], a, vb[0], vb[1]);
          mma16816<T>(o[2 * dp + 1], a, vb[2], vb[3]);
        }
      }
      // Normalise and store (rows past Nq are padding).
      const float inv0 = 1.f / l0, inv1 = 1.f / l1;
      T* out = static_cast<T*>(p.out) + b * p.so[0] + h * p.so[1];
      const int r0 = q0 + g, r1 = q0 + g + 8;
#pragma unroll
      for (int j = 0; j < DT; ++j) {
        const int col = 8 * j + 2 * c;
        if (r0 < nq)
          *reinterpret_cast<uint32_t*>(out + int64_t(r0) * p.so[2] + col) =
              pack_pair<T>(o[j][0] * inv0, o[j][1] * inv0);
        if (r1 < nq)
          *reinterpret_cast<uint32_t*>(out + int64_t(r1) * p.so[2] + col) =
              pack_pair<T>(o[j][2] * inv1, o[j][3] * inv1);
      }
    }

    // The last warp done with this item refills the stage.
    __syncwarp();
    if (lane == 0) {
      const uint32_t done = atomic_add_acq_rel(smem_addr(&count[s]), 1u);
      if (done == uint32_t(W - 1)) {
        count[s] = 0;
        if (i + kStages < my_items) {
          ItemCursor at;
          at.init(int(blockIdx.x) + (i + kStages) * gstep, L);
          fence_proxy_async_smem();
          issue(i + kStages, at);
        }
      }
    }
  }
}

int key_tile(int64_t nk) {
  return nk <= 32 ? 32 : nk <= 64 ? 64 : nk <= 80 ? 80 : 128;
}

template <typename T, int D, int NKP, int PARTS, int NTV>
cudaError_t launch_t(const RbfProblem& p, cudaStream_t stream) {
  const int64_t qmax = p.Nq < 128 ? p.Nq : 128;
  const int W = static_cast<int>((qmax + 15) / 16);
  SmallLaunch L;
  L.qr = 16 * W;
  L.nqb = static_cast<int>((p.Nq + L.qr - 1) / L.qr);
  L.H = static_cast<int>(p.H);
  L.n_items = static_cast<int>(p.B * p.H * L.nqb);
  L.k_off = align1k(L.qr * D * 2);
  L.v_off = L.k_off + align1k(NKP * D * 2);
  L.stage_bytes = L.v_off + align1k(NKP * D * 2);
  auto smem_for = [](int stage_bytes) {
    return 1024 + size_t(kStages) * stage_bytes + size_t(kStages) * NKP * 4 +
           kStages * (8 + 4);
  };
  const size_t smem = smem_for(L.stage_bytes);
  // The attribute is set once, for the largest query block (128 rows).
  const size_t smem_max =
      smem_for(align1k(128 * D * 2) + 2 * align1k(NKP * D * 2));
  CUtensorMap tq, tk, tv;
  if (!make_tile_map(&tq, p.q, p.dtype, p.B, p.H, p.Nq, D, p.sq, L.qr, D) ||
      !make_tile_map(&tk, p.k, p.dtype, p.B, p.H, p.Nk, D, p.sk, NKP, D) ||
      !make_tile_map(&tv, p.v, p.dtype, p.B, p.H, p.Nk, D, p.sv, NKP, D))
    return cudaErrorInvalidValue;
  auto kern = rbf_small_kernel<T, D, NKP, PARTS, NTV>;
  static std::atomic<int> configured[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  if (dev < 0 || dev >= 64 || !configured[dev].load()) {
    cudaError_t err = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
        static_cast<int>(smem_max));
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < 64) configured[dev].store(1);
  }
  int per_sm = 0;
  cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      &per_sm, kern, 32 * W, smem);
  if (err != cudaSuccess) return err;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  int64_t blocks = int64_t(device_sm_count()) * per_sm;
  if (blocks > L.n_items) blocks = L.n_items;
  return launch_pdl(kern, dim3(static_cast<unsigned>(blocks)), dim3(32 * W),
                    smem, stream, tq, tk, tv, p, L);
}

// The key-term split: two threads per key when the CTA has at least two
// threads per key of the tile.
template <typename T, int D, int NKP>
cudaError_t launch_k(const RbfProblem& p, cudaStream_t stream) {
  const int64_t qmax = p.Nq < 128 ? p.Nq : 128;
  const int64_t threads = 32 * ((qmax + 15) / 16);
  // The last 8-key tile is all padding when Nk <= NKP - 8.
  const bool trim = VECTRA_SMALL_TRIM_KEYS && p.Nk <= NKP - 8;
  if (VECTRA_SMALL_SPLIT_KEYS && threads >= 2 * NKP)
    return trim ? launch_t<T, D, NKP, 2, NKP / 8 - 1>(p, stream)
                : launch_t<T, D, NKP, 2, NKP / 8>(p, stream);
  return trim ? launch_t<T, D, NKP, 1, NKP / 8 - 1>(p, stream)
              : launch_t<T, D, NKP, 1, NKP / 8>(p, stream);
}

template <typename T, int D>
cudaError_t launch_d(const RbfProblem& p, cudaStream_t stream) {
  switch (key_tile(p.Nk)) {
    case 32:
      return launch_k<T, D, 32>(p, stream);
    case 64:
      return launch_k<T, D, 64>(p, stream);
    case 80:
      return launch_k<T, D, 80>(p, stream);
    default:
      return launch_k<T, D, 128>(p, stream);
  }
}

template <typename T>
cudaError_t launch_dtype(const RbfProblem& p, cudaStream_t stream) {
  return p.D == 32 ? launch_d<T, 32>(p, stream) : launch_d<T, 64>(p, stream);
}

bool aligned(const void* ptr, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0;
}

}  // namespace

bool small_supports(const RbfProblem& p) {
  if (p.dtype != VECTRA_BF16 && p.dtype != VECTRA_F16) return false;
  if (p.D != p.Dv || (p.D != 32 && p.D != 64)) return false;
  if (p.Nk < 1 || p.Nk > 128 || p.Nq < 2) return false;
  if (p.B * p.H * ((p.Nq + 127) / 128) > (int64_t(1) << 30)) return false;
  if (p.B > (int64_t(1) << 30) || p.H > (int64_t(1) << 30) ||
      p.Nq > (int64_t(1) << 30))
    return false;
  // TMA: 16-byte aligned bases and strides, unit inner stride.
  const void* bases[3] = {p.q, p.k, p.v};
  const int64_t* strides[3] = {p.sq, p.sk, p.sv};
  for (int t = 0; t < 3; ++t) {
    if (!aligned(bases[t], 16) || strides[t][3] != 1) return false;
    for (int d = 0; d < 3; ++d)
      if ((strides[t][d] * 2) % 16 != 0 || strides[t][d] < 0) return false;
  }
  // Output: 4-byte stores of element pairs.
  if (p.so[3] != 1 || !aligned(p.out, 4)) return false;
  if (p.so[0] % 2 || p.so[1] % 2 || p.so[2] % 2) return false;
  return true;
}

cudaError_t launch_small(const RbfProblem& p, cudaStream_t stream) {
  if (!tensor_maps_available()) return cudaErrorNotSupported;
  return p.dtype == VECTRA_BF16 ? launch_dtype<__nv_bfloat16>(p, stream)
                                : launch_dtype<__half>(p, stream);
}

}  // namespace vectra
