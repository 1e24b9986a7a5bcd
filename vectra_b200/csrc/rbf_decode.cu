// rbf_decode.cu: RBF attention for one query per plane (Nq == 1), the
// serving shape (a property scored against its Lk
// comparables). HBM-bound: every byte of K and V is read exactly once.
//
// Design (B200):
//  * Persistent grid, one block per SM, W warps per block. Each warp owns a
//    ring of `ns` shared-memory stages and streams work items (plane, key
//    chunk of KC keys) through it with untiled bulk copies
//    (cp.async.bulk, TMA engine) completing on per-stage mbarriers, so many
//    kilobytes per SM stay in flight without registers holding them.
//  * Key chunks whose bias is -inf are not fetched: the warp reads the bias
//    first and copies only rows [lo, hi] of the chunk that hold a finite
//    bias (the variable-comparable-count config reads ~half the bytes).
//  * Lane j owns keys j, j+32, ...: it forms sum_d (q_d - k_d)^2 from its
//    own key row. Lanes walk the row's 16-byte chunks in a lane-rotated
//    order, so the eight lanes of each shared-memory phase hit eight
//    distinct bank groups (rows are contiguous, so no swizzle is possible).
//  * Softmax over a chunk is exact (max, exp2, sum with warp shuffles);
//    chunks combine online with the reference's safe-max rule. P.V: lane
//    owns DV/32 output columns and walks the chunk's value rows.
//  * Norms are never materialised; the q row is converted to float32 once
//    per plane into a bank-friendly split layout.
#include "rbf_common.cuh"

namespace vectra {
namespace {

template <typename T, int D_, int DV_, int KC_>
struct DecodeCfg {
  static constexpr int D = D_, DV = DV_, KC = KC_;
  static constexpr int ES = sizeof(T);
  static constexpr int E = 16 / ES;            // elements per 16-byte chunk
  static constexpr int C = D * ES / 16;        // chunks per key row
  static constexpr int QB = D * ES;            // bytes of the q row
  static constexpr int KB = KC * D * ES;       // bytes of a key chunk
  static constexpr int VB = KC * DV * ES;      // bytes of a value chunk
  static constexpr int STAGE = QB + KB + VB;
  static constexpr int VE = DV / 32;           // output columns per lane
  static constexpr int KPL = KC / 32;          // keys per lane
  static constexpr int ROT_DIV = C >= 8 ? 1 : 8 / C;
  static_assert(D * ES % 16 == 0, "key rows must be whole 16-byte chunks");
  static_assert(DV % 32 == 0 && KC % 32 == 0, "lane mapping");
  static_assert((C & (C - 1)) == 0, "chunk count must be a power of two");

  // Per-warp shared memory: stages, per-stage bias (exp2 domain) and key
  // range, the float32 q row, the chunk's probabilities, the mbarriers;
  // rounded up to 128 bytes so every warp's stages start 128-byte aligned.
  __host__ __device__ static size_t warp_bytes(int ns) {
    const size_t raw = size_t(ns) * STAGE + size_t(ns) * KC * 4 +
                       size_t(ns) * 16 + D * 4 + KC * 4 + size_t(ns) * 8;
    return (raw + 127) & ~size_t(127);
  }
};

// E elements of a 16-byte chunk as float.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& raw, float* f);
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& raw, float* f) {
  f[0] = __uint_as_float(raw.x);
  f[1] = __uint_as_float(raw.y);
  f[2] = __uint_as_float(raw.z);
  f[3] = __uint_as_float(raw.w);
}
template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& raw,
                                                        float* f) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& raw, float* f) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h2 = *reinterpret_cast<const __half2*>(&w[i]);
    float2 f2 = __half22float2(h2);
    f[2 * i] = f2.x;
    f[2 * i + 1] = f2.y;
  }
}

// VE consecutive elements starting at `ptr` (VE * sizeof(T) bytes aligned).
template <typename T, int VE>
__device__ __forceinline__ void load_slice(const uint8_t* ptr, float* f) {
  const T* t = reinterpret_cast<const T*>(ptr);
  if constexpr (VE * sizeof(T) == 16) {
    unpack16<T>(*reinterpret_cast<const uint4*>(ptr), f);
  } else if constexpr (VE * sizeof(T) == 8) {
    const uint2 raw = *reinterpret_cast<const uint2*>(ptr);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < VE; ++i) f[i] = to_f32(e[i]);
  } else if constexpr (VE * sizeof(T) == 4) {
    const uint32_t raw = *reinterpret_cast<const uint32_t*>(ptr);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < VE; ++i) f[i] = to_f32(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < VE; ++i) f[i] = to_f32(t[i]);
  }
}

template <typename T, int VE>
__device__ __forceinline__ void store_slice(T* dst, const float* f) {
  if constexpr (VE * sizeof(T) == 4 || VE * sizeof(T) == 8 ||
                VE * sizeof(T) == 16) {
    union {
      T e[VE];
      uint32_t w[VE * sizeof(T) / 4];
    } u;
#pragma unroll
    for (int i = 0; i < VE; ++i) u.e[i] = from_f32<T>(f[i]);
    if constexpr (VE * sizeof(T) == 4) {
      *reinterpret_cast<uint32_t*>(dst) = u.w[0];
    } else if constexpr (VE * sizeof(T) == 8) {
      *reinterpret_cast<uint2*>(dst) = make_uint2(u.w[0], u.w[1]);
    } else {
      *reinterpret_cast<uint4*>(dst) =
          make_uint4(u.w[0], u.w[1], u.w[2], u.w[3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < VE; ++i) dst[i] = from_f32<T>(f[i]);
  }
}

template <typename T, int D, int DV, int KC>
__global__ void __launch_bounds__(256, 1)
    rbf_decode_kernel(RbfProblem p, int ns, int64_t n_planes, int k_rows_contig,
                      int v_rows_contig) {
  using Cfg = DecodeCfg<T, D, DV, KC>;
  constexpr int ES = Cfg::ES, E = Cfg::E, C = Cfg::C, QB = Cfg::QB;
  constexpr int KPL = Cfg::KPL, VE = Cfg::VE;
  extern __shared__ __align__(128) uint8_t smem[];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = blockDim.x >> 5;
  const int64_t gw = int64_t(blockIdx.x) * W + warp;
  const int64_t nw = int64_t(gridDim.x) * W;
  if (gw >= n_planes) return;  // warps are independent: no block barrier

  uint8_t* base = smem + size_t(warp) * Cfg::warp_bytes(ns);
  uint8_t* stages = base;
  float* meta_bias = reinterpret_cast<float*>(base + size_t(ns) * Cfg::STAGE);
  int* meta_rng = reinterpret_cast<int*>(meta_bias + ns * KC);
  float* q32 = reinterpret_cast<float*>(meta_rng + 4 * ns);
  float* pvals = q32 + D;
  uint64_t* bars = reinterpret_cast<uint64_t*>(pvals + KC);

  const T* __restrict__ gq = static_cast<const T*>(p.q);
  const T* __restrict__ gk = static_cast<const T*>(p.k);
  const T* __restrict__ gv = static_cast<const T*>(p.v);
  T* __restrict__ gout = static_cast<T*>(p.out);
  const bool has_bias = p.bias != nullptr;
  const uint64_t stream_policy = l2_evict_first_policy();

  const int nchunks = static_cast<int>((p.Nk + KC - 1) / KC);
  const int64_t my_planes = (n_planes - 1 - gw) / nw + 1;
  const int64_t n_items = my_planes * nchunks;

  if (lane == 0) {
    for (int s = 0; s < ns; ++s) mbar_init(smem_addr(&bars[s]), 1);
    fence_barrier_init();
  }
  __syncwarp();

  // Starts the copies of work item `it` into stage `s`.
  auto issue = [&](int64_t it, int s) {
    const int64_t pi = it / nchunks;
    const int chunk = static_cast<int>(it - pi * nchunks);
    const int64_t plane = gw + pi * nw;
    const int64_t b = plane / p.H, h = plane - (plane / p.H) * p.H;
    const int64_t kbase = int64_t(chunk) * KC;
    const int cnt = static_cast<int>(p.Nk - kbase < KC ? p.Nk - kbase : KC);
    int lo = 0, hi = cnt - 1;
    if (has_bias) {
      lo = KC;
      hi = -1;
#pragma unroll
      for (int t = 0; t < KPL; ++t) {
        const int j = lane + 32 * t;
        const float bv =
            j < cnt ? load_bias(p, b, h, kbase + j) * kLog2e : kNegInf;
        meta_bias[s * KC + j] = bv;
        const unsigned live = __ballot_sync(0xffffffffu, bv != kNegInf);
        if (live) {
          lo = min(lo, 32 * t + __ffs(live) - 1);
          hi = max(hi, 32 * t + 31 - __clz(live));
        }
      }
    }
    if (lane == 0) {
      meta_rng[4 * s] = lo;
      meta_rng[4 * s + 1] = hi;
    }
    const int nrows = hi >= lo ? hi - lo + 1 : 0;
    const uint32_t bar = smem_addr(&bars[s]);
    uint8_t* st = stages + size_t(s) * Cfg::STAGE;
    if (lane == 0) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(bar, QB + nrows * (D + DV) * ES);
      bulk_g2s(smem_addr(st), gq + b * p.sq[0] + h * p.sq[1], QB, bar,
               stream_policy);
    }
    __syncwarp();
    if (nrows > 0) {
      const T* k0 = gk + b * p.sk[0] + h * p.sk[1] + (kbase + lo) * p.sk[2];
      const T* v0 = gv + b * p.sv[0] + h * p.sv[1] + (kbase + lo) * p.sv[2];
      uint8_t* kd = st + QB + size_t(lo) * D * ES;
      uint8_t* vd = st + QB + Cfg::KB + size_t(lo) * DV * ES;
      if (k_rows_contig) {
        if (lane == 0)
          bulk_g2s(smem_addr(kd), k0, nrows * D * ES, bar, stream_policy);
      } else {
        for (int r = lane; r < nrows; r += 32)
          bulk_g2s(smem_addr(kd + size_t(r) * D * ES), k0 + r * p.sk[2],
                   D * ES, bar, stream_policy);
      }
      if (v_rows_contig) {
        if (lane == 0)
          bulk_g2s(smem_addr(vd), v0, nrows * DV * ES, bar, stream_policy);
      } else {
        for (int r = lane; r < nrows; r += 32)
          bulk_g2s(smem_addr(vd + size_t(r) * DV * ES), v0 + r * p.sv[2],
                   DV * ES, bar, stream_policy);
      }
    }
  };

  const int64_t prologue = n_items < ns ? n_items : ns;
  for (int64_t it = 0; it < prologue; ++it) issue(it, static_cast<int>(it));

  float g2 = 0.f, m = kNegInf, l = 0.f;
  float acc[VE];
  int64_t it = 0;
  bool failed = false;
  const int rot = lane / Cfg::ROT_DIV;

  for (; it < n_items; ++it) {
    const int s = static_cast<int>(it % ns);
    const uint32_t bar = smem_addr(&bars[s]);
    if (!mbar_wait(bar, static_cast<uint32_t>((it / ns) & 1), p.err)) {
      failed = true;
      break;
    }
    const int64_t pi = it / nchunks;
    const int chunk = static_cast<int>(it - pi * nchunks);
    const int64_t plane = gw + pi * nw;
    const int64_t b = plane / p.H, h = plane - (plane / p.H) * p.H;
    const uint8_t* st = stages + size_t(s) * Cfg::STAGE;
    const int lo = meta_rng[4 * s], hi = meta_rng[4 * s + 1];

    if (chunk == 0) {
      g2 = load_scale(p, b, h) * kLog2e;
      m = kNegInf;
      l = 0.f;
#pragma unroll
      for (int e = 0; e < VE; ++e) acc[e] = 0.f;
      // q32 split layout: element e of chunk ch at [(e / 4) * C + ch][e % 4].
      const T* sq = reinterpret_cast<const T*>(st);
      for (int d = lane; d < D; d += 32) {
        const int ch = d / E, e = d - (d / E) * E;
        q32[((e >> 2) * C + ch) * 4 + (e & 3)] = to_f32(sq[d]);
      }
      __syncwarp();
    }

    // Squared distances of this lane's keys.
    float dist[KPL];
#pragma unroll
    for (int t = 0; t < KPL; ++t) dist[t] = 0.f;
    const uint8_t* ks = st + QB;
#pragma unroll
    for (int cc = 0; cc < C; ++cc) {
      const int ch = (cc + rot) & (C - 1);
      float qv[E];
#pragma unroll
      for (int pp = 0; pp < E / 4; ++pp) {
        const float4 t4 =
            *reinterpret_cast<const float4*>(&q32[(pp * C + ch) * 4]);
        qv[4 * pp] = t4.x;
        qv[4 * pp + 1] = t4.y;
        qv[4 * pp + 2] = t4.z;
        qv[4 * pp + 3] = t4.w;
      }
#pragma unroll
      for (int t = 0; t < KPL; ++t) {
        const int j = lane + 32 * t;
        const uint4 raw = *reinterpret_cast<const uint4*>(
            ks + size_t(j) * D * ES + ch * 16);
        float kf[E];
        unpack16<T>(raw, kf);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float diff = qv[e] - kf[e];
          dist[t] = fmaf(diff, diff, dist[t]);
        }
      }
    }

    // Exact softmax of the chunk, merged online into (m, l, acc).
    float sc[KPL];
    float cmax = kNegInf;
#pragma unroll
    for (int t = 0; t < KPL; ++t) {
      const int j = lane + 32 * t;
      const float bv = has_bias ? meta_bias[s * KC + j] : 0.f;
      sc[t] = (j >= lo && j <= hi) ? fmaf(-g2, dist[t], bv) : kNegInf;
      cmax = fmaxf(cmax, sc[t]);
    }
    cmax = warp_max(cmax);
    const float m_new = fmaxf(m, cmax);
    const float safe = (m_new == kNegInf) ? 0.f : m_new;
    const float alpha = fast_exp2(m - safe);
    float psum = 0.f;
#pragma unroll
    for (int t = 0; t < KPL; ++t) {
      const float pr = fast_exp2(sc[t] - safe);
      pvals[lane + 32 * t] = pr;
      psum += pr;
    }
    psum = warp_sum(psum);
    l = fmaf(l, alpha, psum);
    m = m_new;
    __syncwarp();

#pragma unroll
    for (int e = 0; e < VE; ++e) acc[e] *= alpha;
    const uint8_t* vs = st + QB + Cfg::KB + size_t(lane) * VE * ES;
    int j = lo;
    for (; j + 3 <= hi; j += 4) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float pj = pvals[j + u];
        float vf[VE];
        load_slice<T, VE>(vs + size_t(j + u) * DV * ES, vf);
#pragma unroll
        for (int e = 0; e < VE; ++e) acc[e] = fmaf(pj, vf[e], acc[e]);
      }
    }
    for (; j <= hi; ++j) {
      const float pj = pvals[j];
      float vf[VE];
      load_slice<T, VE>(vs + size_t(j) * DV * ES, vf);
#pragma unroll
      for (int e = 0; e < VE; ++e) acc[e] = fmaf(pj, vf[e], acc[e]);
    }
    __syncwarp();  // every lane is done with stage s and pvals

    if (chunk == nchunks - 1) {
      // Fully masked rows: l == 0 and acc == 0, so 0 * inf = NaN as in
      // the reference.
      const float inv = 1.f / l;
      float o[VE];
#pragma unroll
      for (int e = 0; e < VE; ++e) o[e] = acc[e] * inv;
      store_slice<T, VE>(gout + b * p.so[0] + h * p.so[1] + lane * VE, o);
    }
    if (it + ns < n_items) issue(it + ns, s);
  }

  if (failed) {
    // Drain what is still in flight (bounded) before the block exits.
    for (int64_t r = it + 1; r < n_items && r < it + ns; ++r)
      mbar_wait(smem_addr(&bars[r % ns]), static_cast<uint32_t>((r / ns) & 1),
                p.err);
  }
}

template <typename T, int D, int DV>
struct DecodeLauncher {
  static constexpr int KC_RAW = 16384 / ((D + DV) * int(sizeof(T)));
  static constexpr int KC = KC_RAW >= 128 ? 128 : (KC_RAW >= 64 ? 64 : 32);
  using Cfg = DecodeCfg<T, D, DV, KC>;

  static cudaError_t launch(const RbfProblem& p, cudaStream_t stream) {
    const int ns = 2;
    const size_t per_warp = Cfg::warp_bytes(ns);
    const size_t budget = 227 * 1024;
    int warps = static_cast<int>(budget / per_warp);
    if (warps > 8) warps = 8;
    if (warps < 1) return cudaErrorInvalidConfiguration;
    const int64_t n_planes = p.B * p.H;
    int64_t blocks = (n_planes + warps - 1) / warps;
    const int64_t cap = device_sm_count();
    if (blocks > cap) blocks = cap;
    const size_t smem = per_warp * warps;
    auto kern = rbf_decode_kernel<T, D, DV, KC>;
    cudaError_t err = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
        static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    const int k_contig = p.sk[2] == D;
    const int v_contig = p.sv[2] == DV;
    kern<<<static_cast<unsigned>(blocks), warps * 32, smem, stream>>>(
        p, ns, n_planes, k_contig, v_contig);
    return cudaGetLastError();
  }
};

template <typename T>
cudaError_t dispatch_t(const RbfProblem& p, cudaStream_t stream, bool dry) {
  const int64_t d = p.D, dv = p.Dv;
  if (d != dv) return cudaErrorNotSupported;
  if constexpr (sizeof(T) == 2) {
    if (d == 32) return dry ? cudaSuccess : DecodeLauncher<T, 32, 32>::launch(p, stream);
    if (d == 64) return dry ? cudaSuccess : DecodeLauncher<T, 64, 64>::launch(p, stream);
    if (d == 128) return dry ? cudaSuccess : DecodeLauncher<T, 128, 128>::launch(p, stream);
  } else {
    if (d == 32) return dry ? cudaSuccess : DecodeLauncher<T, 32, 32>::launch(p, stream);
    if (d == 64) return dry ? cudaSuccess : DecodeLauncher<T, 64, 64>::launch(p, stream);
  }
  return cudaErrorNotSupported;
}

cudaError_t dispatch(const RbfProblem& p, cudaStream_t stream, bool dry) {
  switch (p.dtype) {
    case VECTRA_F32:
      return dispatch_t<float>(p, stream, dry);
    case VECTRA_F16:
      return dispatch_t<__half>(p, stream, dry);
    default:
      return dispatch_t<__nv_bfloat16>(p, stream, dry);
  }
}

bool aligned16(const void* ptr) {
  return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0;
}

}  // namespace

bool decode_supports(const RbfProblem& p) {
  if (p.Nq != 1 || p.Nk < 1) return false;
  if (dispatch(p, nullptr, /*dry=*/true) != cudaSuccess) return false;
  const int64_t es = p.dtype == VECTRA_F32 ? 4 : 2;
  // Bulk copies move whole rows: unit innermost stride and 16-byte aligned
  // row starts for q, k and v.
  if (p.sq[3] != 1 || p.sk[3] != 1 || p.sv[3] != 1) return false;
  if (!aligned16(p.q) || !aligned16(p.k) || !aligned16(p.v)) return false;
  for (int i = 0; i < 2; ++i)
    if ((p.sq[i] * es) % 16 || (p.sk[i] * es) % 16 || (p.sv[i] * es) % 16)
      return false;
  if ((p.sk[2] * es) % 16 || (p.sv[2] * es) % 16) return false;
  // Output: each lane stores Dv/32 consecutive elements.
  if (p.so[3] != 1 || !aligned16(p.out)) return false;
  if ((p.so[0] * es) % 16 || (p.so[1] * es) % 16) return false;
  return true;
}

cudaError_t launch_decode(const RbfProblem& p, cudaStream_t stream) {
  return dispatch(p, stream, /*dry=*/false);
}

}  // namespace vectra
