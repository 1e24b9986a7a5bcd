// rbf_small_tc.cu: RBF attention for planes whose queries and keys each fit
// one tile (Nq <= 96, Nk <= 128 - D), on the 5th-generation tensor cores.
// This is the compiled price model's attention site (benchmark config 5:
// per site B=1024, H=8, Nq=Nk=65, D=32, q/k/v strided views of one
// projection, models/price_transformer/spatial_attention.py:68-88); the
// softmax and masking rules are those of the mma.sync kernel (rbf_small.cu)
// and of the reference kernel (spatial_rbf_attention.py:120-166).
//
// Work item: one (b, h) plane. Persistent CTAs, one per SM, 16 warps:
//  * warp 3, one elected lane: TMA producer. For each plane, Q (Nq rows
//    rounded up to 16), K and V (NKP rows) as boxes of 4-D tensor maps over
//    the caller's strides, into a ring of stages (swizzled over the 64- or
//    128-byte row, the canonical UMMA K-major layout; rows past Nq / Nk
//    arrive as zeros).
//  * warp 7: allocates 512 TMEM columns = 4 plane slots of 128 columns
//    (S in the first NKP, overlaid by P as bf16/f16 pairs; O in the last
//    D); one elected lane (elect.sync) issues the MMAs.
//    S = Q K^T is one M=128 x N=NKP tcgen05.mma per 16 dims with both
//    operands in shared memory (Q rows past the box are whatever follows
//    it in shared memory: they only produce S rows nobody reads). O = P V
//    takes P from TMEM (the TS form) and V from shared memory (MN-major).
//    Order: QK(0..3), then PV(i) followed by QK(i+4). MMAs of one thread run
//    in order, so QK(i+4) overwrites slot i % 4's S/P after PV(i) read P.
//  * warps 11 and 15: key terms (b_j - g ||k_j||^2) log2(e) of alternate
//    planes, one lane per key, from the staged K tile; -inf for padded or
//    masked keys. A plane's scale and bias loads are issued while the
//    warp works on its previous plane.
//  * softmax group x = 0..3 (warps 4x + q, q < ceil(Nq / 32)): planes
//    x, x + 4, ... through TMEM slot x. Thread = query row = TMEM lane
//    32q + lane: the S row into registers, logits 2 g log2(e) S_j + t_j
//    (the row-constant -g ||q||^2 cancels in the softmax), exact row max
//    (all keys are in the tile), P = exp2(logit - max) rounded to the input
//    type into TMEM, then after PV the O row / sum, stored to global memory.
//    A row whose keys are all masked ends as 0/0 = NaN, the reference's
//    rule (kernels/vectra_kernels/reference.py:146-152).
// Plane slot x's O is rewritten by PV(i + 4) only after the group has read
// O(i): the group arrives on P(i + 4)'s barrier after its epilogue of i.
// Measured (config 5, B200): 48.1 us per site against 45.7 for the mma.sync
// kernel (rbf_small.cu), so it runs only when forced
// (VECTRA_FLAG_FORCE_SMALL_TC). Traced with clock64 per role and plane, one
// plane per M=128 tile leaves the tensor core ~8% busy and makes each plane
// a serial chain (S -> softmax -> P -> P V -> epilogue) through one of four
// TMEM slots: the four softmax groups fall into lockstep pairs and each
// SMSP idles between chains; removing every exp2 saved only 13%.
// Every mbarrier wait is bounded (error word + early exit); before the
// teardown the producer waits for the loads it issued and the MMA lane for
// the MMAs it issued, so no copy or MMA is in flight when TMEM is freed.
#include <algorithm>
#include <atomic>
#include <type_traits>

#include "rbf_common.cuh"
#include "tcgen05.cuh"

namespace vectra {
namespace {

using namespace tc;

constexpr int kThreads = 512;   // 16 warps
constexpr int kGroups = 4;      // TMEM plane slots = softmax groups
constexpr int kSlotCols = 128;  // TMEM columns per slot: S/P, then O
constexpr int kTmemCols = kGroups * kSlotCols;
constexpr int kProducerWarp = 3;
constexpr int kMmaWarp = 7;
constexpr int kKeyWarp0 = 11;   // and kKeyWarp0 + 4
constexpr int kKeyWarps = 2;
constexpr int kMaxStages = 16;

struct SmallTcLaunch {
  int n_planes;     // B * H
  int H;
  int quads;        // softmax warps per group: ceil(Nq / 32)
  int stages;
  int stage_bytes;  // Q box | K | V
  int k_off;
  int v_off;
  int off_terms;    // float[stages][NKP]
  int off_bar;      // mbarriers, then the TMEM address word
  int tx_bytes;     // bytes of one stage's three boxes
};

// Byte offset of 16-byte chunk `chunk` of row `row` in a TMA tile whose rows
// are RB bytes, swizzled over the row (SWIZZLE_128B / SWIZZLE_64B: address
// bits [7, 7 + log2(RB / 16)) are XORed into the chunk index bits [4, ...)).
template <int RB>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  static_assert(RB == 64 || RB == 128, "row bytes");
  const int x = RB == 128 ? (row & 7) : ((row >> 1) & 3);
  return uint32_t(row * RB + ((chunk ^ x) << 4));
}

// Orders later uses of N registers after a preceding tcgen05.wait::ld
// (emits no instruction).
template <int N>
__device__ __forceinline__ void regs_tie(uint32_t* r) {
  static_assert(N % 8 == 0, "registers");
#pragma unroll
  for (int i = 0; i < N; i += 8)
    asm volatile(""
                 : "+r"(r[i]), "+r"(r[i + 1]), "+r"(r[i + 2]), "+r"(r[i + 3]),
                   "+r"(r[i + 4]), "+r"(r[i + 5]), "+r"(r[i + 6]),
                   "+r"(r[i + 7])
                 :
                 : "memory");
}

// NKP: keys per tile (the MMA's N, a multiple of 16); NV: the S columns the
// softmax reads (Nk rounded up to 8, <= NKP); P is zero past NV.
template <typename T, int D, int NKP, int NV>
__global__ void __launch_bounds__(kThreads, 1)
    rbf_small_tc_kernel(const __grid_constant__ CUtensorMap tq,
                        const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, RbfProblem p,
                        SmallTcLaunch L) {
  static_assert(D == 32 || D == 64, "head width");
  static_assert(NKP % 16 == 0 && NKP + D <= kSlotCols, "slot columns");
  static_assert(NV % 8 == 0 && NV <= NKP, "valid columns");
  constexpr int RB = D * 2;                       // bytes per row
  constexpr uint32_t LAYOUT = RB == 128 ? 2 : 4;  // SWIZZLE_128B / _64B
  constexpr int FMT = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t IDESC_QK = f16_idesc(FMT, 128, NKP, 0);
  constexpr uint32_t IDESC_PV = f16_idesc(FMT, 128, D, 1);
  constexpr int NB = (NKP + 31) / 32;             // keys per key-warp lane
  constexpr uint32_t kOCol = kSlotCols - D;       // O: the slot's last D
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  float* terms = reinterpret_cast<float*>(smem + L.off_terms);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.off_bar);
  const int NS = L.stages;
  // Barriers: kv_full[s], kv_empty[s], nk_full[s], then per slot s_full,
  // p_full, o_full, then drain.
  auto kv_full = [&](int s) { return smem_addr(&bars[s]); };
  auto kv_empty = [&](int s) { return smem_addr(&bars[NS + s]); };
  auto nk_full = [&](int s) { return smem_addr(&bars[2 * NS + s]); };
  auto s_full = [&](int x) { return smem_addr(&bars[3 * NS + x]); };
  auto p_full = [&](int x) { return smem_addr(&bars[3 * NS + 4 + x]); };
  auto o_full = [&](int x) { return smem_addr(&bars[3 * NS + 8 + x]); };
  const uint32_t bar_drain = smem_addr(&bars[3 * NS + 12]);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(&bars[3 * NS + 13]);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = static_cast<int>(p.Nk);
  const int nq = static_cast<int>(p.Nq);
  // Plane i of this CTA is global plane blockIdx.x + i * gridDim.x.
  const int my = L.n_planes > int(blockIdx.x)
                     ? (L.n_planes - 1 - int(blockIdx.x)) / int(gridDim.x) + 1
                     : 0;
  auto plane_bh = [&](int i, int& b, int& h) {
    const int pl = int(blockIdx.x) + i * int(gridDim.x);
    b = pl / L.H;
    h = pl - b * L.H;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
      mbar_init(nk_full(s), 1);
    }
    for (int x = 0; x < kGroups; ++x) {
      mbar_init(s_full(x), 1);
      mbar_init(p_full(x), uint32_t(L.quads));
      mbar_init(o_full(x), 1);
    }
    mbar_init(bar_drain, 1);
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_addr(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  allow_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dependency_wait();  // before any global access
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int issued = 0;
      for (int i = 0; i < my; ++i) {
        const int s = i % NS;
        ok = mbar_wait(kv_empty(s), uint32_t(((i / NS) & 1) ^ 1), p.err);
        if (!ok) break;
        int b, h;
        plane_bh(i, b, h);
        const uint32_t st = sbase + uint32_t(s * L.stage_bytes);
        mbar_arrive_expect_tx(kv_full(s), uint32_t(L.tx_bytes));
        tma_load_4d(st, &tq, kv_full(s), 0, 0, h, b);
        tma_load_4d(st + L.k_off, &tk, kv_full(s), 0, 0, h, b);
        tma_load_4d(st + L.v_off, &tv, kv_full(s), 0, 0, h, b);
        issued = i + 1;
      }
      // The loads issued last have landed before the CTA exits (on an error
      // path some may not have been consumed).
      for (int i = std::max(0, issued - NS); i < issued; ++i)
        if (!mbar_wait(kv_full(i % NS), uint32_t((i / NS) & 1), p.err)) break;
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------- MMA issuer
    if (elect_one()) {
      // K-major Q and K: 8-row groups RB * 8 bytes apart (SBO); a 16-dim
      // k-step is 32 bytes along the swizzled row. MN-major V: 8-key groups
      // RB * 8 bytes apart, one swizzle atom across its D columns; 16 keys
      // per k-step. The descriptor's start field holds addr >> 4, so the
      // descriptor of base + off is the base's plus off >> 4.
      const uint64_t dq0 = swz_desc(sbase, 16, 8 * RB, LAYOUT);
      const uint64_t dk0 = swz_desc(sbase + L.k_off, 16, 8 * RB, LAYOUT);
      const uint64_t dv0 = swz_desc(sbase + L.v_off, NKP * RB, 8 * RB, LAYOUT);
      auto qk = [&](int i) {
        const int x = i % kGroups;
        const uint64_t so = uint64_t(((i % NS) * L.stage_bytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma(tmem + uint32_t(x * kSlotCols), dq0 + so + uint64_t(kk * 2),
                 dk0 + so + uint64_t(kk * 2), IDESC_QK, kk > 0 ? 1u : 0u);
        tc_commit(s_full(x));
      };
      auto pv = [&](int i) {
        const int x = i % kGroups;
        const uint32_t s_tm = tmem + uint32_t(x * kSlotCols);
        const uint64_t so = uint64_t(((i % NS) * L.stage_bytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < NKP / 16; ++kk)
          tc_mma_ts(s_tm + kOCol, s_tm + uint32_t(kk * 8),
                    dv0 + so + uint64_t((kk * 16 * RB) >> 4), IDESC_PV,
                    kk > 0 ? 1u : 0u);
        tc_commit(o_full(x));
        tc_commit(kv_empty(i % NS));  // Q, K and V of plane i are read
      };
      int j = 0;  // the next plane whose S = Q K^T is issued
      for (; j < my && j < kGroups; ++j) {
        ok = mbar_wait(kv_full(j % NS), uint32_t((j / NS) & 1), p.err);
        if (!ok) break;
        tc_fence_after();
        qk(j);
      }
      for (int i = 0; i < my && ok; ++i) {
        ok = mbar_wait(p_full(i % kGroups), uint32_t((i / kGroups) & 1),
                       p.err);
        if (!ok) break;
        tc_fence_after();
        pv(i);
        if (j < my) {
          ok = mbar_wait(kv_full(j % NS), uint32_t((j / NS) & 1), p.err);
          if (!ok) break;
          tc_fence_after();
          qk(j);
          ++j;
        }
      }
      // Every MMA issued above has completed before the teardown.
      tc_commit(bar_drain);
      mbar_wait(bar_drain, 0, p.err);
    }
  } else if (warp == kKeyWarp0 || warp == kKeyWarp0 + 4) {
    // ----------------------------------------------------------- key terms
    // The scale and bias of a warp's next plane are loaded (as raw bits)
    // while it works on the current one: traced on B200, their
    // global-memory latency, exposed once per plane, set the pace of the
    // whole kernel.
    uint32_t gamma_next = 0, bias_next[NB];
    auto prefetch = [&](int i) {
      int b, h;
      plane_bh(i, b, h);
      gamma_next = load_scale_bits(p, b, h);
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        const int j = lane + 32 * t;
        bias_next[t] =
            (p.bias != nullptr && j < nk) ? load_bias_bits(p, b, h, j) : 0u;
      }
    };
    const int first = warp == kKeyWarp0 ? 0 : 1;
    if (first < my) prefetch(first);
    for (int i = first; i < my; i += kKeyWarps) {
      const int s = i % NS;
      const uint32_t gamma_bits = gamma_next;
      uint32_t bias_bits[NB];
#pragma unroll
      for (int t = 0; t < NB; ++t) bias_bits[t] = bias_next[t];
      if (i + kKeyWarps < my) prefetch(i + kKeyWarps);
      ok = mbar_wait(kv_full(s), uint32_t((i / NS) & 1), p.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const uint8_t* ktile = smem + s * L.stage_bytes + L.k_off;
      const float gamma = bias_bits_to_f32(gamma_bits, p.scale_dtype);
#pragma unroll
      for (int t = 0; t < NB; ++t) {
        const int j = lane + 32 * t;
        if (j < NKP) {
          float v = kNegInf;
          if (j < nk) {
            float ax = 0.f, ay = 0.f;
#pragma unroll
            for (int c = 0; c < RB / 16; ++c) {
              const uint4 raw =
                  *reinterpret_cast<const uint4*>(ktile + swz<RB>(j, c));
              const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float lo, hi;
                if constexpr (FMT == 1) {
                  lo = __uint_as_float(w[e] << 16);
                  hi = __uint_as_float(w[e] & 0xffff0000u);
                } else {
                  const float2 f =
                      __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
                  lo = f.x;
                  hi = f.y;
                }
                ax = fmaf(lo, lo, ax);
                ay = fmaf(hi, hi, ay);
              }
            }
            const float bias =
                p.bias != nullptr ? bias_bits_to_f32(bias_bits[t], p.bias_dtype)
                                  : 0.f;
            if (bias != kNegInf) v = (bias - gamma * (ax + ay)) * kLog2e;
          }
          terms[s * NKP + j] = v;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(nk_full(s));
    }
  } else if ((warp & 3) < L.quads) {
    // ------------------------------------------- softmax group x, quadrant q
    const int x = warp >> 2, q = warp & 3;
    const uint32_t s_tm =
        tmem + (uint32_t(q * 32) << 16) + uint32_t(x * kSlotCols);
    const uint32_t o_tm = s_tm + kOCol;
    const int row = q * 32 + lane;
    uint32_t scale_next = 0;  // the next plane's scale, loaded a plane ahead
    if (x < my) {
      int b, h;
      plane_bh(x, b, h);
      scale_next = load_scale_bits(p, b, h);
    }
    for (int i = x, n = 0; i < my; i += kGroups, ++n) {
      const int s = i % NS;
      int b, h;
      plane_bh(i, b, h);
      const uint32_t scale_bits = scale_next;
      if (i + kGroups < my) {
        int b1, h1;
        plane_bh(i + kGroups, b1, h1);
        scale_next = load_scale_bits(p, b1, h1);
      }
      ok = mbar_wait(s_full(x), uint32_t(n & 1), p.err) &&
           mbar_wait(nk_full(s), uint32_t((i / NS) & 1), p.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[NV];
      tmem_ld_cols<NV>(s_tm, sv);
      tmem_wait_ld();
      regs_tie<NV>(sv);
      // Logits in place, row max over four independent accumulators.
      const float* tj = terms + s * NKP;
      const float g2 =
          2.f * bias_bits_to_f32(scale_bits, p.scale_dtype) * kLog2e;
      const uint64_t g2x2 = f2pk(g2, g2);
      float mxa = kNegInf, mxb = kNegInf, mxc = kNegInf, mxd = kNegInf;
#pragma unroll
      for (int j = 0; j < NV; j += 8) {
        const float4 n4 = *reinterpret_cast<const float4*>(tj + j);
        const float4 m4 = *reinterpret_cast<const float4*>(tj + j + 4);
        const float2 l01 = f2upk(ffma2(
            g2x2, f2pk(__uint_as_float(sv[j]), __uint_as_float(sv[j + 1])),
            f2pk(n4.x, n4.y)));
        const float2 l23 = f2upk(ffma2(
            g2x2, f2pk(__uint_as_float(sv[j + 2]), __uint_as_float(sv[j + 3])),
            f2pk(n4.z, n4.w)));
        const float2 l45 = f2upk(ffma2(
            g2x2, f2pk(__uint_as_float(sv[j + 4]), __uint_as_float(sv[j + 5])),
            f2pk(m4.x, m4.y)));
        const float2 l67 = f2upk(ffma2(
            g2x2, f2pk(__uint_as_float(sv[j + 6]), __uint_as_float(sv[j + 7])),
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
      const float ref = mx == kNegInf ? 0.f : mx;
      const uint64_t negref2 = f2pk(-ref, -ref);
      // P = exp2(logit - max), rounded to T in pairs, over the S columns.
      uint32_t pw[NKP / 2];
      uint64_t suma = 0, sumb = 0;
#pragma unroll
      for (int j = 0; j < NV; j += 4) {
        const float2 x01 = f2upk(fadd2(
            f2pk(__uint_as_float(sv[j]), __uint_as_float(sv[j + 1])), negref2));
        const float2 x23 = f2upk(fadd2(
            f2pk(__uint_as_float(sv[j + 2]), __uint_as_float(sv[j + 3])),
            negref2));
        const float e0 = fast_exp2(x01.x), e1 = fast_exp2(x01.y);
        const float e2 = fast_exp2(x23.x), e3 = fast_exp2(x23.y);
        suma = fadd2(suma, f2pk(e0, e1));
        sumb = fadd2(sumb, f2pk(e2, e3));
        pw[j / 2] = pack2<T>(e0, e1);
        pw[j / 2 + 1] = pack2<T>(e2, e3);
      }
#pragma unroll
      for (int w = NV / 2; w < NKP / 2; ++w) pw[w] = 0u;
      tmem_st_cols<NKP / 2>(s_tm, pw);
      const float2 sa = f2upk(suma), sb = f2upk(sumb);
      const float l = (sa.x + sa.y) + (sb.x + sb.y);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full(x));
      // Epilogue: O / l for this row.
      ok = mbar_wait(o_full(x), uint32_t(n & 1), p.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t ov[D];
      tmem_ld_cols<D>(o_tm, ov);
      tmem_wait_ld();
      regs_tie<D>(ov);
      if (row < nq) {
        const float inv = 1.f / l;
        T* orow = static_cast<T*>(p.out) + b * p.so[0] + h * p.so[1] +
                  int64_t(row) * p.so[2];
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          uint4 u;
          u.x = pack2<T>(__uint_as_float(ov[8 * c]) * inv,
                         __uint_as_float(ov[8 * c + 1]) * inv);
          u.y = pack2<T>(__uint_as_float(ov[8 * c + 2]) * inv,
                         __uint_as_float(ov[8 * c + 3]) * inv);
          u.z = pack2<T>(__uint_as_float(ov[8 * c + 4]) * inv,
                         __uint_as_float(ov[8 * c + 5]) * inv);
          u.w = pack2<T>(__uint_as_float(ov[8 * c + 6]) * inv,
                         __uint_as_float(ov[8 * c + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + 8 * c) = u;
        }
      }
    }
  }

  // Teardown: every TMEM access is done before the allocating warp frees it.
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int align1k(int x) { return (x + 1023) & ~1023; }

template <typename T, int D, int NKP, int NV>
cudaError_t launch_t(const RbfProblem& p, cudaStream_t stream) {
  constexpr int RB = D * 2;
  SmallTcLaunch L;
  const int qbox = static_cast<int>((p.Nq + 15) / 16 * 16);
  L.n_planes = static_cast<int>(p.B * p.H);
  L.H = static_cast<int>(p.H);
  L.quads = static_cast<int>((p.Nq + 31) / 32);
  L.k_off = qbox * RB;
  L.v_off = L.k_off + NKP * RB;
  L.stage_bytes = align1k(L.v_off + NKP * RB);
  L.tx_bytes = (qbox + 2 * NKP) * RB;
  // The S MMA reads 128 Q rows from each stage's base: the last stage's
  // read may run past it, into the key terms and barriers after the ring
  // (never past the allocation).
  const int tail_need = 128 * RB - L.stage_bytes;
  const int fixed = (3 * kMaxStages + 13) * 8 + 16;  // barriers + TMEM word
  const int budget = 227 * 1024 - 1024;               // minus the alignment
  int stages = 1;
  auto layout = [&](int ns) {
    const int terms = ns * NKP * 4;
    const int after = std::max(terms + fixed, tail_need);
    return ns * L.stage_bytes + after;
  };
  while (stages < kMaxStages && layout(stages + 1) <= budget) ++stages;
  // The MMA lane issues S = Q K^T for kGroups planes before the first
  // O = P V: the ring must hold them all, or it would wait for a stage that
  // only a later P V frees.
  if (stages < kGroups || layout(stages) > budget)
    return cudaErrorInvalidConfiguration;
  L.stages = stages;
  L.off_terms = stages * L.stage_bytes;
  L.off_bar = L.off_terms + stages * NKP * 4;
  const size_t smem = 1024 + size_t(layout(stages));

  CUtensorMap tq, tk, tv;
  if (!make_tile_map(&tq, p.q, p.dtype, p.B, p.H, p.Nq, D, p.sq, qbox, D) ||
      !make_tile_map(&tk, p.k, p.dtype, p.B, p.H, p.Nk, D, p.sk, NKP, D) ||
      !make_tile_map(&tv, p.v, p.dtype, p.B, p.H, p.Nk, D, p.sv, NKP, D))
    return cudaErrorInvalidValue;
  auto kern = rbf_small_tc_kernel<T, D, NKP, NV>;
  static std::atomic<int> configured[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  if (dev < 0 || dev >= 64 || !configured[dev].load()) {
    const cudaError_t err = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < 64) configured[dev].store(1);
  }
  int64_t blocks = device_sm_count();
  if (blocks > L.n_planes) blocks = L.n_planes;
  return launch_pdl(kern, dim3(static_cast<unsigned>(blocks)),
                    dim3(kThreads), smem, stream, tq, tk, tv, p, L);
}

template <typename T, int D, int NKP>
cudaError_t launch_k(const RbfProblem& p, cudaStream_t stream) {
  // S columns read by the softmax: Nk rounded up to 8 when that trims the
  // tile by 8 keys (65 keys in an 80-key tile: 72 columns).
  if (p.Nk <= NKP - 8) return launch_t<T, D, NKP, NKP - 8>(p, stream);
  return launch_t<T, D, NKP, NKP>(p, stream);
}

// Keys per tile: 32, 64, 80 or 96 for D = 32; 32 or 64 for D = 64.
template <typename T>
cudaError_t launch_dtype(const RbfProblem& p, cudaStream_t stream) {
  if (p.D == 32) {
    if (p.Nk <= 32) return launch_k<T, 32, 32>(p, stream);
    if (p.Nk <= 64) return launch_k<T, 32, 64>(p, stream);
    if (p.Nk <= 80) return launch_k<T, 32, 80>(p, stream);
    return launch_k<T, 32, 96>(p, stream);
  }
  if (p.Nk <= 32) return launch_k<T, 64, 32>(p, stream);
  return launch_k<T, 64, 64>(p, stream);
}

bool aligned(const void* ptr, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0;
}

}  // namespace

bool small_tc_supports(const RbfProblem& p) {
  if (p.dtype != VECTRA_BF16 && p.dtype != VECTRA_F16) return false;
  if (p.D != p.Dv || (p.D != 32 && p.D != 64)) return false;
  if (p.Nq < 2 || p.Nq > 96 || p.Nk < 1 || p.Nk > 128 - p.D) return false;
  if (p.B * p.H > (int64_t(1) << 30) || p.B > (int64_t(1) << 30)) return false;
  // TMA: 16-byte aligned bases and strides, unit inner stride.
  const void* bases[3] = {p.q, p.k, p.v};
  const int64_t* strides[3] = {p.sq, p.sk, p.sv};
  for (int t = 0; t < 3; ++t) {
    if (!aligned(bases[t], 16) || strides[t][3] != 1) return false;
    for (int d = 0; d < 3; ++d)
      if ((strides[t][d] * 2) % 16 != 0 || strides[t][d] < 0) return false;
  }
  // Output: 16-byte stores of 8 elements.
  if (p.so[3] != 1 || !aligned(p.out, 16)) return false;
  if (p.so[0] % 8 || p.so[1] % 8 || p.so[2] % 8) return false;
  return true;
}

cudaError_t launch_small_tc(const RbfProblem& p, cudaStream_t stream) {
  if (!tensor_maps_available()) return cudaErrorNotSupported;
  return p.dtype == VECTRA_BF16 ? launch_dtype<__nv_bfloat16>(p, stream)
                                : launch_dtype<__half>(p, stream);
}

}  // namespace vectra
