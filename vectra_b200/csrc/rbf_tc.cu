// rbf_tc.cu: RBF attention on the 5th-generation tensor cores (tcgen05 +
// TMEM) for long sequences (B=16, H=16, Lq=Lk=4096,
// D=128, bf16), a true dense contraction.
//
// Algebra: the row-constant -g*||q||^2 cancels in the softmax, so
//   softmax_j(-g(||q||^2 + ||k_j||^2 - 2 q.k_j) + b_j)
//     = softmax_j(2g q.k_j - g ||k_j||^2 + b_j),
// which is one GEMM (S = Q K^T on the tensor cores) plus a per-key term
// computed from the K tile already in shared memory (no norm pre-pass, unlike
// kernels/vectra_kernels/norm_precompute.py). The reference clamps the
// squared distance at zero (spatial_rbf_attention.py:137); that only matters
// for near-duplicate rows and is within tolerance.
//
// One CTA per (b, h, tile of 128 queries); 8 warps:
//  * warp 0, one lane: TMA producer. Q once, then K and V tiles of 128 keys
//    into a 2-stage ring (128-byte swizzled, the canonical UMMA K-major /
//    MN-major layouts), via 4-D tensor maps over [B, H, N, D] with the
//    caller's strides. No multicast.
//  * warp 1: allocates TMEM (S: 128 columns, O: Dv columns); lane 0 issues
//    the MMAs: S = Q K^T (kind::f16, M=128, N=128, fp32 accumulate in TMEM),
//    then O += P V once the softmax has written P (bf16, swizzled smem).
//    tcgen05.commit signals completion on mbarriers.
//  * warps 4-7 (one thread per query row, matching TMEM lanes 0-127):
//    per key tile, the key norms (thread r: key r, read straight from the
//    swizzled K tile), then tcgen05.ld of the S row, logits in the exp2
//    domain, row max, P = exp2(logit - m) written to smem, running sum.
//    O is rescaled in TMEM only when the row max grew by more than 8 (a
//    factor of 256), the lazy-rescaling rule, so most tiles skip it.
//  * Epilogue: the softmax warps read O from TMEM, divide by the running
//    sum and store their rows.
// Every mbarrier wait is bounded (error word + early exit, no trap).
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <type_traits>

#include "rbf_common.cuh"

namespace vectra {
namespace {

constexpr int kTileM = 128;   // query rows per CTA (TMEM lanes)
constexpr int kTileN = 128;   // keys per tile
constexpr int kStages = 2;    // K/V ring depth
constexpr int kThreads = 256;
constexpr int kSoftmaxWarp0 = 4;
constexpr float kRescaleThreshold = 8.f;  // log2 of the lazy-rescale factor

template <int D>
struct TcCfg {
  static_assert(D == 64 || D == 128, "head width");
  static constexpr int KB = D / 64;                  // 128-byte column blocks
  static constexpr int BLOCK = kTileN * 128;         // one 128-row x 128 B block
  static constexpr int Q_BYTES = kTileM * D * 2;
  static constexpr int K_BYTES = kTileN * D * 2;
  static constexpr int V_BYTES = kTileN * D * 2;
  static constexpr int P_BYTES = kTileM * kTileN * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_KV = OFF_Q + Q_BYTES;     // + s * STAGE
  static constexpr int STAGE = K_BYTES + V_BYTES;    // K then V
  static constexpr int OFF_P = OFF_KV + kStages * STAGE;
  static constexpr int OFF_NK = OFF_P + P_BYTES;     // float[2][128]
  static constexpr int OFF_BAR = OFF_NK + 2 * kTileN * 4;
  static constexpr int NBAR = 8 + 2 * kStages;
  static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_TMEM + 16;
  static constexpr int SMEM_ALLOC = SMEM + 1024;     // for 1024-B alignment
  static constexpr int TMEM_COLS = 256;              // S (128) + O (<= 128)
  static constexpr uint32_t TMEM_O = 128;            // column of O
};

// ---------------------------------------------------------------------------
// PTX wrappers (tcgen05, TMA, descriptors).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::
          "r"(dst_smem),
      "r"(ncols)
      : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(bar)
      : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16, fp32 accumulate.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc,
                                       uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, "
      "%7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, "
      "%21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, "
      "%7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, "
      "%21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
      "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])),
      "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
      "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])),
      "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
      "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
      "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// 4-D tiled TMA load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap,
                                            uint32_t bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1),
      "r"(c2), "r"(c3)
      : "memory");
}
// Named barrier over `count` threads that also ANDs `pred` across them, so
// a failure seen by any thread becomes every thread's decision.
__device__ __forceinline__ bool named_barrier_and(int id, int count,
                                                  bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred q, p;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(pred)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 format:
// start >> 4 in bits 0-13, LBO >> 4 in 16-29, SBO >> 4 in 32-45, version 1
// in bits 46-47, layout type 2 = SWIZZLE_128B in bits 61-63).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo,
                                               uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3fff);
  d |= uint64_t((lbo >> 4) & 0x3fff) << 16;
  d |= uint64_t((sbo >> 4) & 0x3fff) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

// Instruction descriptor of kind::f16 with fp32 accumulation.
__host__ __device__ constexpr uint32_t f16_idesc(int ab_format, int m, int n,
                                                 int b_mn_major) {
  return (1u << 4) | (uint32_t(ab_format) << 7) | (uint32_t(ab_format) << 10) |
         (uint32_t(b_mn_major) << 16) | (uint32_t(n >> 3) << 17) |
         (uint32_t(m >> 4) << 24);
}

struct TcParams {
  int n_qtiles;       // ceil(Nq / 128)
  int n_ktiles;       // ceil(Nk / 128)
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    rbf_tc_kernel(const __grid_constant__ CUtensorMap tq,
                  const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, RbfProblem p,
                  TcParams P) {
  using Cfg = TcCfg<D>;
  constexpr int FMT = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t IDESC_QK = f16_idesc(FMT, kTileM, kTileN, 0);
  constexpr uint32_t IDESC_PV = f16_idesc(FMT, kTileM, D, 1);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  // Barriers: 0 q_full, 1 s_full, 2 s_free, 3 p_full, 4 pv_done,
  // 8.. kv_full[kStages], 8 + kStages.. kv_empty[kStages].
  const uint32_t bar_q = smem_addr(&bars[0]);
  const uint32_t bar_s_full = smem_addr(&bars[1]);
  const uint32_t bar_s_free = smem_addr(&bars[2]);
  const uint32_t bar_p_full = smem_addr(&bars[3]);
  const uint32_t bar_pv_done = smem_addr(&bars[4]);
  auto bar_kv_full = [&](int s) { return smem_addr(&bars[8 + s]); };
  auto bar_kv_empty = [&](int s) { return smem_addr(&bars[8 + kStages + s]); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::OFF_TMEM);
  float* nk_smem = reinterpret_cast<float*>(smem + Cfg::OFF_NK);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x % P.n_qtiles;
  const int plane = blockIdx.x / P.n_qtiles;
  const int H = static_cast<int>(p.H);
  const int b = plane / H, h = plane - b * H;
  const int q0 = qt * kTileM;
  const int nk = static_cast<int>(p.Nk);
  const int n_tiles = P.n_ktiles;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    mbar_init(bar_s_full, 1);
    mbar_init(bar_s_free, 4);
    mbar_init(bar_p_full, 4);
    mbar_init(bar_pv_done, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_kv_full(s), 1);
      mbar_init(bar_kv_empty(s), 1);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem;
  const uint32_t tmem_o = tmem + Cfg::TMEM_O;
  bool ok = true;

  if (warp == 0) {
    // ------------------------------------------------------------- producer
    if (lane == 0) {
      mbar_arrive_expect_tx(bar_q, Cfg::Q_BYTES);
      for (int kb = 0; kb < Cfg::KB; ++kb)
        tma_load_4d(sbase + Cfg::OFF_Q + kb * Cfg::BLOCK, &tq, bar_q, kb * 64,
                    q0, h, b);
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int s = t % kStages;
        ok = mbar_wait(bar_kv_empty(s), uint32_t(((t / kStages) & 1) ^ 1),
                       p.err);
        if (!ok) break;
        const uint32_t st = sbase + Cfg::OFF_KV + s * Cfg::STAGE;
        mbar_arrive_expect_tx(bar_kv_full(s), Cfg::STAGE);
        for (int kb = 0; kb < Cfg::KB; ++kb) {
          tma_load_4d(st + kb * Cfg::BLOCK, &tk, bar_kv_full(s), kb * 64,
                      t * kTileN, h, b);
          tma_load_4d(st + Cfg::K_BYTES + kb * Cfg::BLOCK, &tv,
                      bar_kv_full(s), kb * 64, t * kTileN, h, b);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      ok = mbar_wait(bar_q, 0, p.err);
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int s = t % kStages;
        const uint32_t st = sbase + Cfg::OFF_KV + s * Cfg::STAGE;
        ok = mbar_wait(bar_kv_full(s), uint32_t((t / kStages) & 1), p.err);
        if (ok && t > 0) ok = mbar_wait(bar_s_free, uint32_t((t - 1) & 1), p.err);
        if (!ok) break;
        tc_fence_after();
        // S = Q K^T: K = D in steps of 16 (32 bytes inside a 128-byte row).
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * Cfg::BLOCK + (kk & 3) * 32;
          tc_mma(tmem_s, sw128_desc(sbase + Cfg::OFF_Q + off, 16, 1024),
                 sw128_desc(st + off, 16, 1024), IDESC_QK, kk > 0);
        }
        tc_commit(bar_s_full);
        ok = mbar_wait(bar_p_full, uint32_t(t & 1), p.err);
        if (!ok) break;
        tc_fence_after();
        // O += P V: K = 128 keys in steps of 16; V is MN-major (dims
        // contiguous): 16 keys = two 8-row groups of 128 B (SBO 1024),
        // 64-dim blocks BLOCK bytes apart (LBO).
#pragma unroll
        for (int kk = 0; kk < kTileN / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * Cfg::BLOCK + (kk & 3) * 32;
          tc_mma(tmem_o, sw128_desc(sbase + Cfg::OFF_P + poff, 16, 1024),
                 sw128_desc(st + Cfg::K_BYTES + kk * 16 * 128, Cfg::BLOCK,
                            1024),
                 IDESC_PV, (t > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(bar_pv_done);
        tc_commit(bar_kv_empty(s));
      }
    }
  } else if (warp >= kSoftmaxWarp0) {
    // --------------------------------------------------- softmax + epilogue
    const int r = threadIdx.x - kSoftmaxWarp0 * 32;  // query row = TMEM lane
    const uint32_t lane_base = uint32_t((warp & 3) * 32) << 16;
    const float g = load_scale(p, b, h) * kLog2e;     // g log2(e)
    const float a2 = 2.f * g;
    float m_used = kNegInf, l = 0.f;
    uint8_t* ptile = smem + Cfg::OFF_P;
    // Every thread runs all n_tiles iterations and every named barrier; after a
    // failed (timed-out) wait, `ok` turns false for the whole warpgroup at
    // the next barrier and the remaining iterations skip their work. Waits
    // are made warp-uniform so tcgen05.ld/st always run convergent.
    for (int t = 0; t < n_tiles; ++t) {
      const int s = t % kStages;
      const uint8_t* ktile = smem + Cfg::OFF_KV + s * Cfg::STAGE;
      float* nkb = nk_smem + (t & 1) * kTileN;
      if (ok) ok = mbar_wait(bar_kv_full(s), uint32_t((t / kStages) & 1), p.err);
      ok = __all_sync(0xffffffffu, ok);
      // Key r's term g log2e ||k_r||^2 - log2e b_r (+inf when masked or
      // past the end). The row's 16-byte chunks are summed in an order
      // rotated by r % 8 so the eight rows of a phase hit distinct banks.
      if (ok) {
        const int key = t * kTileN + r;
        float nv = __int_as_float(0x7f800000);
        if (key < nk) {
          float accx = 0.f, accy = 0.f;
#pragma unroll
          for (int kb = 0; kb < Cfg::KB; ++kb) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint4 raw = *reinterpret_cast<const uint4*>(
                  ktile + kb * Cfg::BLOCK + r * 128 + ((c ^ (r & 7)) << 4));
              const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                float lo, hi;
                if constexpr (FMT == 1) {
                  lo = __uint_as_float(w[i] << 16);
                  hi = __uint_as_float(w[i] & 0xffff0000u);
                } else {
                  const float2 f = __half22float2(
                      *reinterpret_cast<const __half2*>(&w[i]));
                  lo = f.x;
                  hi = f.y;
                }
                accx = fmaf(lo, lo, accx);
                accy = fmaf(hi, hi, accy);
              }
            }
          }
          nv = g * (accx + accy);
          if (p.bias) nv -= load_bias(p, b, h, key) * kLog2e;
        }
        nkb[r] = nv;
      }
      ok = named_barrier_and(1, 128, ok);
      if (!ok) continue;

      ok = mbar_wait(bar_s_full, uint32_t(t & 1), p.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) continue;
      tc_fence_after();
      float sv[kTileN];
#pragma unroll
      for (int c = 0; c < kTileN / 32; ++c)
        tmem_ld32(tmem_s + lane_base + c * 32, sv + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_s_free);  // S may be overwritten
      float mx = kNegInf;
#pragma unroll
      for (int j = 0; j < kTileN; j += 4) {
        const float4 n4 = *reinterpret_cast<const float4*>(nkb + j);
        sv[j] = fmaf(a2, sv[j], -n4.x);
        sv[j + 1] = fmaf(a2, sv[j + 1], -n4.y);
        sv[j + 2] = fmaf(a2, sv[j + 2], -n4.z);
        sv[j + 3] = fmaf(a2, sv[j + 3], -n4.w);
        mx = fmaxf(mx, fmaxf(fmaxf(sv[j], sv[j + 1]),
                             fmaxf(sv[j + 2], sv[j + 3])));
      }
      // P(t-1) consumed and O(t-1) final before P and O are touched.
      if (t > 0) {
        ok = mbar_wait(bar_pv_done, uint32_t((t - 1) & 1), p.err);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) continue;
        tc_fence_after();
      }
      // Lazy rescaling: move this row's reference max only when the max
      // grew by more than 2^8; the warp rescales O if any row moved.
      const bool need = mx > m_used + kRescaleThreshold ||
                        (m_used == kNegInf && mx != kNegInf);
      float factor = 1.f;
      if (need) {
        factor = m_used == kNegInf ? 0.f : fast_exp2(m_used - mx);
        m_used = mx;
        l *= factor;
      }
      if (t > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float ov[32];
          tmem_ld32(tmem_o + lane_base + c * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= factor;
          tmem_st32(tmem_o + lane_base + c * 32, ov);
        }
        tmem_wait_st();
      }
      const float ref = m_used == kNegInf ? 0.f : m_used;
      float lsum = 0.f;
#pragma unroll
      for (int kb = 0; kb < 2; ++kb) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          union {
            T e[8];
            uint4 u;
          } pk8;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float pr = fast_exp2(sv[kb * 64 + c * 8 + e] - ref);
            lsum += pr;
            pk8.e[e] = from_f32<T>(pr);
          }
          *reinterpret_cast<uint4*>(ptile + kb * Cfg::BLOCK + r * 128 +
                                    ((c ^ (r & 7)) << 4)) = pk8.u;
        }
      }
      l += lsum;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p_full);
    }
    // Epilogue: O / l for this row.
    if (ok) ok = mbar_wait(bar_pv_done, uint32_t((n_tiles - 1) & 1), p.err);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      const int qrow = q0 + r;
      const float inv = 1.f / l;
      T* orow = static_cast<T*>(p.out) + b * p.so[0] + h * p.so[1] +
                int64_t(qrow) * p.so[2];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float ov[32];
        tmem_ld32(tmem_o + lane_base + c * 32, ov);
        tmem_wait_ld();
        if (qrow < p.Nq) {
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            union {
              T e[8];
              uint4 u;
            } pk8;
#pragma unroll
            for (int e = 0; e < 8; ++e)
              pk8.e[e] = from_f32<T>(ov[v4 * 8 + e] * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + v4 * 8) = pk8.u;
          }
        }
      }
    }
  }

  // Teardown: every TMEM access is done before the allocating warp frees it.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps and launch.
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr,
                                cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// [B, H, N, D] view with element strides s (s[3] == 1), box 64 x 128.
bool make_map(CUtensorMap* map, const void* base, int dtype, int64_t B,
              int64_t H, int64_t N, int64_t D, const int64_t* s) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int64_t es = 2;
  cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(N), cuuint64_t(H),
                        cuuint64_t(B)};
  cuuint64_t strides[3] = {cuuint64_t(s[2] * es), cuuint64_t(s[1] * es),
                           cuuint64_t(s[0] * es)};
  // Broadcast or degenerate strides: give size-1 dimensions a valid stride.
  if (N == 1) strides[0] = cuuint64_t(D * es + 15) / 16 * 16;
  if (H == 1) strides[1] = strides[0] * N;
  if (B == 1) strides[2] = strides[1] * H;
  cuuint32_t box[4] = {64, cuuint32_t(kTileN), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map,
                        dtype == VECTRA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int D>
cudaError_t launch_t(const RbfProblem& p, cudaStream_t stream) {
  using Cfg = TcCfg<D>;
  CUtensorMap tq, tk, tv;
  if (encode_fn() == nullptr) return cudaErrorNotSupported;
  if (!make_map(&tq, p.q, p.dtype, p.B, p.H, p.Nq, D, p.sq) ||
      !make_map(&tk, p.k, p.dtype, p.B, p.H, p.Nk, D, p.sk) ||
      !make_map(&tv, p.v, p.dtype, p.B, p.H, p.Nk, D, p.sv))
    return cudaErrorInvalidValue;
  TcParams P;
  P.n_qtiles = static_cast<int>((p.Nq + kTileM - 1) / kTileM);
  P.n_ktiles = static_cast<int>((p.Nk + kTileN - 1) / kTileN);
  const int64_t blocks = int64_t(P.n_qtiles) * p.B * p.H;
  auto kern = rbf_tc_kernel<T, D>;
  static std::atomic<int> configured[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  if (dev < 0 || dev >= 64 || !configured[dev].load()) {
    cudaError_t err = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_ALLOC);
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < 64) configured[dev].store(1);
  }
  kern<<<static_cast<unsigned>(blocks), kThreads, Cfg::SMEM_ALLOC, stream>>>(
      tq, tk, tv, p, P);
  return cudaGetLastError();
}

bool aligned16(const void* ptr) {
  return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0;
}

}  // namespace

bool tc_supports(const RbfProblem& p) {
  if (p.dtype != VECTRA_BF16 && p.dtype != VECTRA_F16) return false;
  if (p.D != p.Dv || (p.D != 64 && p.D != 128)) return false;
  if (p.Nq < 128 || p.Nk < 128) return false;
  if (p.B * p.H * ((p.Nq + 127) / 128) > (int64_t(1) << 31) - 1) return false;
  if (p.Nq > (int64_t(1) << 31) - 1 || p.Nk > (int64_t(1) << 31) - 1)
    return false;
  // TMA: unit innermost stride, 16-byte aligned bases and strides.
  if (p.sq[3] != 1 || p.sk[3] != 1 || p.sv[3] != 1 || p.so[3] != 1)
    return false;
  if (!aligned16(p.q) || !aligned16(p.k) || !aligned16(p.v) ||
      !aligned16(p.out))
    return false;
  // Strides of size-1 dimensions are never used (the tensor map rewrites
  // them); the others must be non-negative multiples of 16 bytes.
  const int64_t sizes_q[3] = {p.B, p.H, p.Nq}, sizes_k[3] = {p.B, p.H, p.Nk};
  for (int i = 0; i < 3; ++i) {
    if (sizes_q[i] > 1 && (p.sq[i] < 0 || (p.sq[i] * 2) % 16)) return false;
    if (sizes_k[i] > 1 && (p.sk[i] < 0 || (p.sk[i] * 2) % 16 || p.sv[i] < 0 ||
                           (p.sv[i] * 2) % 16))
      return false;
    if (sizes_q[i] > 1 && (p.so[i] * 2) % 16) return false;
  }
  return true;
}

cudaError_t launch_tc(const RbfProblem& p, cudaStream_t stream) {
  if (p.dtype == VECTRA_BF16)
    return p.D == 64 ? launch_t<__nv_bfloat16, 64>(p, stream)
                     : launch_t<__nv_bfloat16, 128>(p, stream);
  return p.D == 64 ? launch_t<__half, 64>(p, stream)
                   : launch_t<__half, 128>(p, stream);
}

}  // namespace vectra
