// rbf_tc.cu: RBF attention on the 5th-generation tensor cores (tcgen05 +
// TMEM) for long sequences (benchmark config 4: B=16, H=16, Lq=Lk=4096,
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
// One CTA per (b, h, 256 queries) = two query tiles A and B of 128 rows,
// 12 warps in three warpgroups:
//  * WG0 (warps 0-3) and WG1 (warps 4-7): softmax of tile A and tile B, one
//    thread per query row (TMEM lanes 0-127). Per key tile: S is read from
//    TMEM twice (row max, then exp2), P = exp2(logit - m) is written back
//    into TMEM over the S columns already read (bf16 pairs), and O is
//    rescaled in TMEM only when the row max grew by more than 8 (a factor
//    of 256, the lazy-rescaling rule).
//  * warp 8, one elected lane: TMA producer. Q (both tiles) once, then K and
//    V tiles of 128 keys into a 2-stage ring (128-byte swizzled, the
//    canonical UMMA K-major / MN-major layouts) via 4-D tensor maps over
//    [B, H, N, D] with the caller's strides; each CTA loads its own tiles.
//  * warp 9: allocates all 512 TMEM columns (S_A, S_B, O_A, O_B); one lane
//    issues the MMAs, ping-ponging the tiles so the tensor core works on
//    one tile while the other's softmax runs:
//      QK_A(0) QK_B(0) | PV_A(t) QK_A(t+1) PV_B(t) QK_B(t+1) | ...
//    S = Q K^T is kind::f16 with both operands in shared memory; O += P V
//    takes P from TMEM (the TS form) and V from shared memory. MMAs of one
//    thread execute in order, so QK_X(t+1) overwriting S_X (and P_X) runs
//    after PV_X(t) has read P_X.
//  * warps 10-11: key terms g log2e ||k_j||^2 - log2e b_j for each K tile
//    (64 threads x 2 keys, read straight from the swizzled tile), published
//    per stage through an mbarrier.
//  * Epilogue: each softmax warpgroup reads its O from TMEM, divides by the
//    running sum and stores its rows.
// Every mbarrier wait is bounded (error word + early exit, no trap).
#include <atomic>
#include <mutex>
#include <type_traits>

#include "rbf_common.cuh"
#include "tcgen05.cuh"

namespace vectra {
namespace {

constexpr int kTileM = 128;   // query rows per tile (TMEM lanes)
constexpr int kTilesQ = 2;    // query tiles per CTA (A and B)
constexpr int kTileN = 128;   // keys per tile
constexpr int kStages = 2;    // K/V ring depth
constexpr int kThreads = 384;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kNormWarp0 = 10;
constexpr int kNormThreads = 64;
constexpr float kRescaleThreshold = 8.f;  // log2 of the lazy-rescale factor
// Register split (setmaxnreg): the two softmax warpgroups hold a whole S row
// (128 values) in registers; the producer / MMA / key-term warpgroup needs
// few. The launch gives every thread kLaunchRegs; the split must not exceed
// that total (checked on the host against the compiled kernel before any
// launch), or setmaxnreg.inc would wait for registers that never come.
constexpr int kSoftmaxRegs = 200;
constexpr int kOtherRegs = 104;

template <int D>
struct TcCfg {
  static_assert(D == 64 || D == 128, "head width");
  static constexpr int KB = D / 64;                  // 128-byte column blocks
  static constexpr int BLOCK = kTileN * 128;         // 128 rows x 128 B
  static constexpr int Q_TILE = kTileM * D * 2;
  static constexpr int Q_BYTES = kTilesQ * Q_TILE;
  static constexpr int K_BYTES = kTileN * D * 2;
  static constexpr int V_BYTES = kTileN * D * 2;
  static constexpr int OFF_Q = 0;                    // + x * Q_TILE
  static constexpr int OFF_KV = OFF_Q + Q_BYTES;     // + s * STAGE
  static constexpr int STAGE = K_BYTES + V_BYTES;    // K then V
  static constexpr int OFF_NK = OFF_KV + kStages * STAGE;  // float[kStages][128]
  static constexpr int OFF_BAR = OFF_NK + kStages * kTileN * 4;
  static constexpr int NBAR = 16;
  static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_TMEM + 16;
  static constexpr int SMEM_ALLOC = SMEM + 1024;     // for 1024-B alignment
  static constexpr int TMEM_COLS = 512;
  // TMEM columns: S_A, S_B (128 each; P_X overlays the first 64 of S_X),
  // then O_A, O_B.
  __host__ __device__ static constexpr uint32_t s_col(int x) {
    return uint32_t(x) * 128;
  }
  __host__ __device__ static constexpr uint32_t o_col(int x) {
    return 256 + uint32_t(x) * 128;
  }
};

using namespace tc;

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
  // Barriers: 0 q_full; 1, 2 s_full[A, B]; 3, 4 p_full[A, B];
  // 5, 6 o_final[A, B]; 8 + s kv_full[s]; 10 + s kv_empty[s];
  // 12 + s nk_full[s].
  const uint32_t bar_q = smem_addr(&bars[0]);
  auto bar_s_full = [&](int x) { return smem_addr(&bars[1 + x]); };
  auto bar_p_full = [&](int x) { return smem_addr(&bars[3 + x]); };
  auto bar_o_final = [&](int x) { return smem_addr(&bars[5 + x]); };
  auto bar_kv_full = [&](int s) { return smem_addr(&bars[8 + s]); };
  auto bar_kv_empty = [&](int s) { return smem_addr(&bars[10 + s]); };
  auto bar_nk_full = [&](int s) { return smem_addr(&bars[12 + s]); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::OFF_TMEM);
  float* nk_smem = reinterpret_cast<float*>(smem + Cfg::OFF_NK);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x % P.n_qtiles;
  const int plane = blockIdx.x / P.n_qtiles;
  const int H = static_cast<int>(p.H);
  const int b = plane / H, h = plane - b * H;
  const int q0 = qt * (kTilesQ * kTileM);
  const int nk = static_cast<int>(p.Nk);
  const int n_tiles = P.n_ktiles;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int x = 0; x < kTilesQ; ++x) {
      mbar_init(bar_s_full(x), 1);
      mbar_init(bar_p_full(x), 4);
      mbar_init(bar_o_final(x), 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_kv_full(s), 1);
      mbar_init(bar_kv_empty(s), 1);
      mbar_init(bar_nk_full(s), kNormThreads / 32);
    }
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_addr(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  allow_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dependency_wait();  // before any global access
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp >= kProducerWarp) {
  setmaxnreg_dec<kOtherRegs>();
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------- producer
    if (elect_one()) {
      mbar_arrive_expect_tx(bar_q, Cfg::Q_BYTES);
      for (int x = 0; x < kTilesQ; ++x)
        for (int kb = 0; kb < Cfg::KB; ++kb)
          tma_load_4d(sbase + Cfg::OFF_Q + x * Cfg::Q_TILE + kb * Cfg::BLOCK,
                      &tq, bar_q, kb * 64, q0 + x * kTileM, h, b);
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
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------- MMA issuer
    if (elect_one()) {
      // Descriptors of the tile bases, built once: a descriptor's start
      // address field holds addr >> 4 (14 bits; shared-memory offsets stay
      // below 256 KB), so the descriptor of base + off (off a multiple of
      // 16) is the base's plus off >> 4, one add per MMA.
      const uint64_t dq0 = sw128_desc(sbase + Cfg::OFF_Q, 16, 1024);
      const uint64_t dk0 = sw128_desc(sbase + Cfg::OFF_KV, 16, 1024);
      const uint64_t dv0 =
          sw128_desc(sbase + Cfg::OFF_KV + Cfg::K_BYTES, Cfg::BLOCK, 1024);
      auto qk = [&](int x, int t) {
        const uint64_t dq = dq0 + uint64_t((x * Cfg::Q_TILE) >> 4);
        const uint64_t dk = dk0 + uint64_t(((t % kStages) * Cfg::STAGE) >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * Cfg::BLOCK + (kk & 3) * 32) >> 4;
          tc_mma(tmem + Cfg::s_col(x), dq + off, dk + off, IDESC_QK, kk > 0);
        }
        tc_commit(bar_s_full(x));
      };
      auto pv = [&](int x, int t) {
        const uint64_t dv = dv0 + uint64_t(((t % kStages) * Cfg::STAGE) >> 4);
        // P_X: bf16 pairs in TMEM over S_X, 8 columns per 16 keys. V is
        // MN-major: 16 keys = two 8-row groups of 128 B (SBO 1024),
        // 64-dim blocks BLOCK bytes apart (LBO).
#pragma unroll
        for (int kk = 0; kk < kTileN / 16; ++kk)
          tc_mma_ts(tmem + Cfg::o_col(x), tmem + Cfg::s_col(x) + kk * 8,
                    dv + uint64_t((kk * 16 * 128) >> 4), IDESC_PV,
                    (t > 0 || kk > 0) ? 1u : 0u);
      };
      ok = mbar_wait(bar_q, 0, p.err);
      if (ok) ok = mbar_wait(bar_kv_full(0), 0, p.err);
      if (ok) {
        tc_fence_after();
        qk(0, 0);
        qk(1, 0);
      }
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int s = t % kStages;
        const bool more = t + 1 < n_tiles;
        const int s1 = (t + 1) % kStages;
        ok = mbar_wait(bar_p_full(0), uint32_t(t & 1), p.err);
        if (ok && more)
          ok = mbar_wait(bar_kv_full(s1), uint32_t(((t + 1) / kStages) & 1),
                         p.err);
        if (!ok) break;
        tc_fence_after();
        pv(0, t);
        if (more) qk(0, t + 1);
        ok = mbar_wait(bar_p_full(1), uint32_t(t & 1), p.err);
        if (!ok) break;
        tc_fence_after();
        pv(1, t);
        tc_commit(bar_kv_empty(s));  // K and V of tile t are no longer read
        if (more) qk(1, t + 1);
      }
      if (ok) {
        tc_commit(bar_o_final(0));
        tc_commit(bar_o_final(1));
      }
    }
  } else if (warp >= kNormWarp0) {
    // ------------------------------------------------------- key terms
    const int th = threadIdx.x - kNormWarp0 * 32;  // 0..63
    const float g = load_scale(p, b, h) * kLog2e;
    for (int t = 0; t < n_tiles && ok; ++t) {
      const int s = t % kStages;
      ok = mbar_wait(bar_kv_full(s), uint32_t((t / kStages) & 1), p.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const uint8_t* ktile = smem + Cfg::OFF_KV + s * Cfg::STAGE;
#pragma unroll
      for (int i = 0; i < kTileN / kNormThreads; ++i) {
        const int r = th + i * kNormThreads;
        const int key = t * kTileN + r;
        float nv = __int_as_float(0x7f800000);  // past the end: masked
        if (key < nk) {
          float accx = 0.f, accy = 0.f;
#pragma unroll
          for (int kb = 0; kb < Cfg::KB; ++kb) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              // Chunk order rotated by r % 8: the eight rows of a phase
              // hit distinct bank groups.
              const uint4 raw = *reinterpret_cast<const uint4*>(
                  ktile + kb * Cfg::BLOCK + r * 128 + ((c ^ (r & 7)) << 4));
              const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
              for (int k2 = 0; k2 < 4; ++k2) {
                float lo, hi;
                if constexpr (FMT == 1) {
                  lo = __uint_as_float(w[k2] << 16);
                  hi = __uint_as_float(w[k2] & 0xffff0000u);
                } else {
                  const float2 f = __half22float2(
                      *reinterpret_cast<const __half2*>(&w[k2]));
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
        nk_smem[s * kTileN + r] = -nv;  // stored negated: logit = a2 S + this
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_nk_full(s));
    }
  }
  } else {
    // --------------------------------------------- softmax, tile x = A/B
    setmaxnreg_inc<kSoftmaxRegs>();
    const int x = warp >> 2;                  // 0: A (warps 0-3), 1: B
    const int r = threadIdx.x & 127;          // query row = TMEM lane
    const uint32_t lane_base = uint32_t((warp & 3) * 32) << 16;
    const uint32_t s_col = tmem + lane_base + Cfg::s_col(x);
    const uint32_t o_col = tmem + lane_base + Cfg::o_col(x);
    const float a2 = 2.f * load_scale(p, b, h) * kLog2e;
    float m_used = kNegInf, l = 0.f;
    for (int t = 0; t < n_tiles && ok; ++t) {
      const int s = t % kStages;
      const float* nkb = nk_smem + s * kTileN;
      ok = mbar_wait(bar_s_full(x), uint32_t(t & 1), p.err) &&
           mbar_wait(bar_nk_full(s), uint32_t((t / kStages) & 1), p.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      // The whole S row into registers (four 32-column loads, one wait),
      // turned into logits a2 * S - nk in place; the row max with four
      // independent accumulators.
      const uint64_t a2x2 = f2pk(a2, a2);
      uint32_t sv[kTileN];
#pragma unroll
      for (int c = 0; c < kTileN / 32; ++c) tmem_ld32u(s_col + c * 32, sv + c * 32);
      tmem_wait_ld_tied(sv);
#pragma unroll
      for (int c = 1; c < kTileN / 32; ++c) regs_tie32(sv + c * 32);
      float mxa = kNegInf, mxb = kNegInf, mxc = kNegInf, mxd = kNegInf;
#pragma unroll
      for (int j = 0; j < kTileN; j += 8) {
        const float4 n4 = *reinterpret_cast<const float4*>(nkb + j);
        const float4 m4 = *reinterpret_cast<const float4*>(nkb + j + 4);
        const float2 l01 = f2upk(ffma2(
            a2x2, f2pk(__uint_as_float(sv[j]), __uint_as_float(sv[j + 1])),
            f2pk(n4.x, n4.y)));
        const float2 l23 = f2upk(ffma2(
            a2x2, f2pk(__uint_as_float(sv[j + 2]), __uint_as_float(sv[j + 3])),
            f2pk(n4.z, n4.w)));
        const float2 l45 = f2upk(ffma2(
            a2x2, f2pk(__uint_as_float(sv[j + 4]), __uint_as_float(sv[j + 5])),
            f2pk(m4.x, m4.y)));
        const float2 l67 = f2upk(ffma2(
            a2x2, f2pk(__uint_as_float(sv[j + 6]), __uint_as_float(sv[j + 7])),
            f2pk(m4.z, m4.w)));
        sv[j] = __float_as_uint(l01.x);
        sv[j + 1] = __float_as_uint(l01.y);
        sv[j + 2] = __float_as_uint(l23.x);
        sv[j + 3] = __float_as_uint(l23.y);
        sv[j + 4] = __float_as_uint(l45.x);
        sv[j + 5] = __float_as_uint(l45.y);
        sv[j + 6] = __float_as_uint(l67.x);
        sv[j + 7] = __float_as_uint(l67.y);
        mxa = fmax3(mxa, l01.x, l01.y);
        mxb = fmax3(mxb, l23.x, l23.y);
        mxc = fmax3(mxc, l45.x, l45.y);
        mxd = fmax3(mxd, l67.x, l67.y);
      }
      const float mx = fmaxf(fmaxf(mxa, mxb), fmaxf(mxc, mxd));
      // Lazy rescaling: move this row's reference max only when the max
      // grew by more than 2^8; the warp rescales O if any of its rows moved.
      // (PV_X(t-1) has completed: QK_X(t) ran after it, in order.)
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
          tmem_ld32(o_col + c * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= factor;
          tmem_st32(o_col + c * 32, ov);
        }
      }
      // P = exp2(logit - m) from the registers, packed to pairs and
      // stored over the S columns (chunk c -> P columns 16c..16c+15).
      const float ref = m_used == kNegInf ? 0.f : m_used;
      const uint64_t negref2 = f2pk(-ref, -ref);
      uint64_t lsum2a = 0, lsum2b = 0;
#pragma unroll
      for (int c = 0; c < kTileN / 32; ++c) {
        uint32_t pp[16];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const int k = c * 32 + j;
          const float2 x01 = f2upk(fadd2(
              f2pk(__uint_as_float(sv[k]), __uint_as_float(sv[k + 1])),
              negref2));
          const float2 x23 = f2upk(fadd2(
              f2pk(__uint_as_float(sv[k + 2]), __uint_as_float(sv[k + 3])),
              negref2));
          const float e0 = fast_exp2(x01.x), e1 = fast_exp2(x01.y);
          const float e2 = fast_exp2(x23.x), e3 = fast_exp2(x23.y);
          lsum2a = fadd2(lsum2a, f2pk(e0, e1));
          lsum2b = fadd2(lsum2b, f2pk(e2, e3));
          pp[j / 2] = pack2<T>(e0, e1);
          pp[j / 2 + 1] = pack2<T>(e2, e3);
        }
        tmem_st16(s_col + c * 16, pp);
      }
      const float2 la = f2upk(lsum2a), lb = f2upk(lsum2b);
      const float lsum = (la.x + la.y) + (lb.x + lb.y);
      l += lsum;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p_full(x));
    }
    // Epilogue: O / l for this row.
    if (ok) ok = mbar_wait(bar_o_final(x), 0, p.err);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      const int qrow = q0 + x * kTileM + r;
      const float inv = 1.f / l;
      T* orow = static_cast<T*>(p.out) + b * p.so[0] + h * p.so[1] +
                int64_t(qrow) * p.so[2];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float ov[32];
        tmem_ld32(o_col + c * 32, ov);
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
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps and launch.
// ---------------------------------------------------------------------------
template <typename T, int D>
cudaError_t launch_t(const RbfProblem& p, cudaStream_t stream) {
  using Cfg = TcCfg<D>;
  CUtensorMap tq, tk, tv;
  if (!tensor_maps_available()) return cudaErrorNotSupported;
  if (!make_tile_map(&tq, p.q, p.dtype, p.B, p.H, p.Nq, D, p.sq, kTileN) ||
      !make_tile_map(&tk, p.k, p.dtype, p.B, p.H, p.Nk, D, p.sk, kTileN) ||
      !make_tile_map(&tv, p.v, p.dtype, p.B, p.H, p.Nk, D, p.sv, kTileN))
    return cudaErrorInvalidValue;
  TcParams P;
  P.n_qtiles = static_cast<int>((p.Nq + kTilesQ * kTileM - 1) /
                               (kTilesQ * kTileM));
  P.n_ktiles = static_cast<int>((p.Nk + kTileN - 1) / kTileN);
  const int64_t blocks = int64_t(P.n_qtiles) * p.B * p.H;
  auto kern = rbf_tc_kernel<T, D>;
  static std::atomic<int> configured[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  if (dev < 0 || dev >= 64 || !configured[dev].load()) {
    // The setmaxnreg split must fit in the registers the block is launched
    // with; a deficit would leave setmaxnreg.inc waiting forever.
    cudaFuncAttributes attr;
    cudaError_t err = cudaFuncGetAttributes(&attr, kern);
    if (err != cudaSuccess) return err;
    if (int64_t(attr.numRegs) * kThreads <
        int64_t(2 * 128) * kSoftmaxRegs + int64_t(128) * kOtherRegs)
      return cudaErrorInvalidConfiguration;
    err = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_ALLOC);
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < 64) configured[dev].store(1);
  }
  return launch_pdl(kern, dim3(static_cast<unsigned>(blocks)), dim3(kThreads),
                    Cfg::SMEM_ALLOC, stream, tq, tk, tv, p, P);
}

bool aligned16(const void* ptr) {
  return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0;
}

}  // namespace

bool tc_supports(const RbfProblem& p) {
  if (p.dtype != VECTRA_BF16 && p.dtype != VECTRA_F16) return false;
  if (p.D != p.Dv || (p.D != 64 && p.D != 128)) return false;
  if (p.Nq < 128 || p.Nk < 128) return false;
  if (p.B * p.H * ((p.Nq + 255) / 256) > (int64_t(1) << 31) - 1) return false;
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
