// rbf_decode_mma.cu: RBF attention for one query per plane (Nq == 1) with
// the dot products on the tensor cores (mma.sync m16n8k16, bf16/f16 in,
// fp32 accumulate). Same work split as rbf_decode.cu (one warp per
// (query, head) plane, a block-shared ring of stages filled by the TMA,
// online softmax across key chunks with warp shuffles), but the per-plane
// arithmetic that made the SIMT kernel issue-bound (~1,700 instructions per
// 64-key plane) becomes 64 MMAs and 32 ldmatrix per plane:
//
//  * S = K q: A = K (keys x dims, from a 128-byte-swizzled TMA tile via
//    ldmatrix), B = q in column 0 of an n8 tile (lanes 0-3), so column 0 of
//    the accumulator holds q.k_j for the 16 keys of an m-tile.
//  * ||k_j||^2: the diagonal of K_m K_m^T per 16-key m-tile. With A = K_m,
//    the B fragments of K_m^T for the two n8 halves are exactly the A
//    registers {a0, a2} and {a1, a3}, so the norms cost two MMAs per
//    (m-tile, k-step) and no extra loads; the diagonal is gathered with one
//    shuffle.
//  * O^T = V^T p: A = V^T via ldmatrix.trans of the value tile, B = p in
//    column 0 (lanes 0-3, bf16/f16, as the reference rounds P to v's dtype
//    before P.V: kernels/vectra_kernels/spatial_rbf_attention.py:163).
//
// Logits are 2 g q.k_j - g ||k_j||^2 + b_j in the exp2 domain (the
// row-constant -g ||q||^2 cancels in the softmax). Keys are fetched in boxes
// of 16 rows; boxes of a chunk whose keys all carry a -inf bias are neither
// fetched nor multiplied. Every wait is bounded.
#include <atomic>

#include "mma_sync.cuh"
#include "rbf_common.cuh"

namespace vectra {
namespace {

constexpr int kWarps = 8;
constexpr int kBoxRows = 16;

template <int D>
struct DmCfg {
  static_assert(D == 64 || D == 128, "head width");
  static constexpr int KB = D / 64;             // 64-dim blocks (128 B rows)
  static constexpr int KC = D == 64 ? 64 : 32;  // keys per chunk
  static constexpr int MT = KC / 16;            // 16-key m-tiles per chunk
  static constexpr int DT = D / 16;             // 16-dim tiles
  static constexpr int BLOCK = KC * 128;        // one 64-dim block, KC rows
  static constexpr int STAGE = 2 * KB * BLOCK;  // K blocks, then V blocks
  static constexpr int QB = D * 2;              // q row bytes
  static constexpr int META = 16 + KC * 4;      // lo, hi, armed | bias[KC]
  static size_t block_bytes(int ns, int warps) {
    return size_t(ns) * (STAGE + QB + META + 8) + 16 +
           size_t(warps) * D * 4 + 1024;
  }
};

struct DmLaunch {
  int ns;
  int n_planes;
  int H;
  int nchunks;
};

template <typename T, int D>
__global__ void __launch_bounds__(32 * kWarps, 1)
    rbf_decode_mma_kernel(const __grid_constant__ CUtensorMap tk,
                          const __grid_constant__ CUtensorMap tv,
                          RbfProblem p, DmLaunch L) {
  using Cfg = DmCfg<D>;
  constexpr int KB = Cfg::KB, KC = Cfg::KC, MT = Cfg::MT, DT = Cfg::DT;
  constexpr int KPL = KC / 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ns = L.ns;
  // Layout: stages | q rows | per-stage meta | mbarriers | per-warp output.
  uint8_t* stages = smem;
  uint8_t* qrows = stages + size_t(ns) * Cfg::STAGE;
  uint8_t* metas = qrows + size_t(ns) * Cfg::QB;
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(metas + size_t(ns) * Cfg::META);
  float* obuf_all = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(bars + ns) + 15) & ~uintptr_t(15));
  auto meta_int = [&](int s) {
    return reinterpret_cast<int*>(metas + size_t(s) * Cfg::META);
  };
  auto meta_bias = [&](int s) {
    return reinterpret_cast<float*>(metas + size_t(s) * Cfg::META + 16);
  };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = blockDim.x >> 5;
  const bool has_bias = p.bias != nullptr;
  const int nk = static_cast<int>(p.Nk);
  const int nchunks = L.nchunks;
  const int n_slots = (L.n_planes - 1 - int(blockIdx.x)) / int(gridDim.x) + 1;
  const int n_items = n_slots * nchunks;
  const T* __restrict__ gq = static_cast<const T*>(p.q);
  T* __restrict__ gout = static_cast<T*>(p.out);
  float* obuf = obuf_all + warp * D;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(smem_addr(&bars[s]), 1);
      meta_int(s)[2] = -1;
    }
    fence_barrier_init();
  }
  allow_dependents();
  __syncthreads();
  grid_dependency_wait();  // before any global access

  // Copies item i into stage i % ns; lane 31 (which never stores output)
  // arms the copies and then publishes "stage s holds item i".
  constexpr int kIssueLane = 31;
  auto issue = [&](int i) {
    const int g = i / nchunks, chunk = i - g * nchunks;
    const int s = i % ns;
    const int plane = int(blockIdx.x) + g * int(gridDim.x);
    const int b = plane / L.H, h = plane - b * L.H;
    const int kbase = chunk * KC;
    const int cnt = min(KC, nk - kbase);
    int lo = 0, hi = cnt - 1;
    if (has_bias) {
      lo = KC;
      hi = -1;
      float* mb = meta_bias(s);
#pragma unroll
      for (int t = 0; t < KPL; ++t) {
        const int j = lane + 32 * t;
        const float bv =
            j < cnt ? load_bias(p, b, h, kbase + j) * kLog2e : kNegInf;
        mb[j] = bv;
        const unsigned live = __ballot_sync(0xffffffffu, bv != kNegInf);
        if (live) {
          lo = min(lo, 32 * t + __ffs(live) - 1);
          hi = max(hi, 32 * t + 31 - __clz(live));
        }
      }
    }
    const int b0 = hi >= lo ? lo / kBoxRows : 0;
    const int nbox = hi >= lo ? hi / kBoxRows - b0 + 1 : 0;
    const uint32_t bar = smem_addr(&bars[s]);
    const uint32_t st = smem_addr(stages + size_t(s) * Cfg::STAGE);
    __syncwarp();
    if (lane == kIssueLane) {
      int* mi = meta_int(s);
      mi[0] = lo;
      mi[1] = hi;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(bar, Cfg::QB + nbox * kBoxRows * 128 * KB * 2);
      bulk_g2s(smem_addr(qrows + size_t(s) * Cfg::QB),
               gq + b * p.sq[0] + h * p.sq[1], Cfg::QB, bar,
               l2_evict_normal_policy());
      for (int bb = b0; bb < b0 + nbox; ++bb) {
        for (int kb = 0; kb < KB; ++kb) {
          const uint32_t off = kb * Cfg::BLOCK + bb * kBoxRows * 128;
          tma_load_4d(st + off, &tk, bar, kb * 64, kbase + bb * kBoxRows, h,
                      b);
          tma_load_4d(st + KB * Cfg::BLOCK + off, &tv, bar, kb * 64,
                      kbase + bb * kBoxRows, h, b);
        }
      }
      st_release_smem(&mi[2], i);
    }
    __syncwarp();
  };

  for (int i = warp; i < ns && i < n_items; i += W) issue(i);

  const int r = lane >> 2, c = lane & 3;
  // ldmatrix row/chunk of this lane for an A tile of K (non-transposed) and
  // of V^T (transposed).
  const int a_row = (lane & 7) + 8 * ((lane >> 3) & 1);
  const int a_chk = lane >> 4;
  const int v_row = (lane & 7) + 8 * (lane >> 4);
  const int v_chk = (lane >> 3) & 1;

  for (int g = warp; g < n_slots; g += W) {
    const int plane = int(blockIdx.x) + g * int(gridDim.x);
    const int b = plane / L.H, h = plane - b * L.H;
    const float g2 = load_scale(p, b, h) * kLog2e;
    const float a2 = 2.f * g2;
    float m = kNegInf, l = 0.f;
    float acc_o[DT][4];
#pragma unroll
    for (int t = 0; t < DT; ++t)
      acc_o[t][0] = acc_o[t][1] = acc_o[t][2] = acc_o[t][3] = 0.f;
    uint32_t bq[DT][2];

    for (int chunk = 0; chunk < nchunks; ++chunk) {
      const int i = g * nchunks + chunk;
      const int s = i % ns;
      if (!wait_smem_equals(&meta_int(s)[2], i, p.err) ||
          !mbar_wait_sleep(smem_addr(&bars[s]), uint32_t((i / ns) & 1),
                           p.err))
        return;  // error recorded; the host reports it
      const int lo = meta_int(s)[0], hi = meta_int(s)[1];
      const uint32_t stk = smem_addr(stages + size_t(s) * Cfg::STAGE);
      const uint32_t stv = stk + KB * Cfg::BLOCK;

      if (chunk == 0) {
        // B fragments of q (column 0 of the n8 tile): lanes 0-3 only.
        const uint32_t* q32 =
            reinterpret_cast<const uint32_t*>(qrows + size_t(s) * Cfg::QB);
#pragma unroll
        for (int kk = 0; kk < DT; ++kk) {
          bq[kk][0] = lane < 4 ? q32[(16 * kk + 2 * lane) / 2] : 0u;
          bq[kk][1] = lane < 4 ? q32[(16 * kk + 2 * lane + 8) / 2] : 0u;
        }
      }
      // Everything this item needs from the stage goes to registers first
      // (K and V^T fragments, this lane's key biases), so the stage is
      // refilled at once instead of after the whole computation.
      bool live[MT];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
        live[mt] = !(16 * mt + 15 < lo || 16 * mt > hi);  // box fetched
      uint32_t ka[MT][DT][4], va[MT][DT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        if (!live[mt]) continue;
        const int key = 16 * mt + a_row;
        const int vkey = 16 * mt + v_row;
#pragma unroll
        for (int kk = 0; kk < DT; ++kk) {
          const int kb = kk >> 2;
          const int ch = 2 * (kk & 3) + a_chk, vch = 2 * (kk & 3) + v_chk;
          ldsm_x4(stk + kb * Cfg::BLOCK + key * 128 + ((ch ^ (key & 7)) << 4),
                  ka[mt][kk]);
          ldsm_x4_t(stv + kb * Cfg::BLOCK + vkey * 128 +
                        ((vch ^ (vkey & 7)) << 4),
                    va[mt][kk]);
        }
      }
      float bias_r[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        bias_r[mt][0] = has_bias ? meta_bias(s)[16 * mt + r] : 0.f;
        bias_r[mt][1] = has_bias ? meta_bias(s)[16 * mt + 8 + r] : 0.f;
      }
      __syncwarp();  // every lane is done with stage s
      if (i + ns < n_items) issue(i + ns);

      // S = K q and the diagonal blocks of K K^T, per 16-key m-tile.
      float acc_s[MT][4], acc_n0[MT][4], acc_n1[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          acc_s[mt][e] = acc_n0[mt][e] = acc_n1[mt][e] = 0.f;
        if (!live[mt]) continue;
#pragma unroll
        for (int kk = 0; kk < DT; ++kk) {
          const uint32_t* a = ka[mt][kk];
          mma16816<T>(acc_s[mt], a, bq[kk][0], bq[kk][1]);
          mma16816<T>(acc_n0[mt], a, a[0], a[2]);
          mma16816<T>(acc_n1[mt], a, a[1], a[3]);
        }
      }

      // Logits of keys 16 mt + r (lo half) and 16 mt + 8 + r (hi half),
      // meaningful in lanes c == 0 (column 0); other lanes hold -inf.
      float lg[MT][2];
      float cmax = kNegInf;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        // Diagonal of the 16x16 block: key 16mt + r sits in lane
        // 4r + r/2 (c0 for even r, c1 for odd); key 16mt + 8 + r likewise
        // in c2/c3 of the second n8 half.
        const float d0 = (r & 1) ? acc_n0[mt][1] : acc_n0[mt][0];
        const float d1 = (r & 1) ? acc_n1[mt][3] : acc_n1[mt][2];
        const int src = 4 * r + (r >> 1);
        const float n_lo = __shfl_sync(0xffffffffu, d0, src);
        const float n_hi = __shfl_sync(0xffffffffu, d1, src);
        const int j0 = 16 * mt + r, j1 = j0 + 8;
        float l0 = fmaf(a2, acc_s[mt][0], -g2 * n_lo);
        float l1 = fmaf(a2, acc_s[mt][2], -g2 * n_hi);
        if (has_bias) {
          l0 += bias_r[mt][0];
          l1 += bias_r[mt][1];
        }
        lg[mt][0] = (c == 0 && j0 >= lo && j0 <= hi) ? l0 : kNegInf;
        lg[mt][1] = (c == 0 && j1 >= lo && j1 <= hi) ? l1 : kNegInf;
        cmax = fmaxf(cmax, fmaxf(lg[mt][0], lg[mt][1]));
      }
      // One butterfly over (max, sum of exp2 relative to that max).
      float lsum = 0.f;
      {
        const float lsafe = (cmax == kNegInf) ? 0.f : cmax;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          lsum += fast_exp2(lg[mt][0] - lsafe) + fast_exp2(lg[mt][1] - lsafe);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, cmax, off);
        const float ol = __shfl_xor_sync(0xffffffffu, lsum, off);
        const float nm = fmaxf(cmax, om);
        const float ns_ = (nm == kNegInf) ? 0.f : nm;
        lsum = lsum * fast_exp2(cmax - ns_) + ol * fast_exp2(om - ns_);
        cmax = nm;
      }
      const float m_new = fmaxf(m, cmax);
      const float safe = (m_new == kNegInf) ? 0.f : m_new;
      const float alpha = fast_exp2(m - safe);
      // lsum is relative to the chunk max; exp2(cmax - safe) is <= 1 and 0
      // for a fully masked chunk (where lsum is 0 too).
      l = fmaf(l, alpha, lsum * fast_exp2(cmax - safe));
      m = m_new;
#pragma unroll
      for (int t = 0; t < DT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc_o[t][e] *= alpha;

      // O^T += V^T p, one 16-key k-step per fetched box.
#pragma unroll
      for (int kk = 0; kk < MT; ++kk) {
        if (!live[kk]) continue;
        const float p_lo = fast_exp2(lg[kk][0] - safe);  // key 16kk + r
        const float p_hi = fast_exp2(lg[kk][1] - safe);  // key 16kk + 8 + r
        const int s0 = 8 * (lane & 3), s1 = s0 + 4;
        const float x0 = __shfl_sync(0xffffffffu, p_lo, s0);
        const float x1 = __shfl_sync(0xffffffffu, p_lo, s1);
        const float x2 = __shfl_sync(0xffffffffu, p_hi, s0);
        const float x3 = __shfl_sync(0xffffffffu, p_hi, s1);
        const uint32_t b0 = lane < 4 ? pack_pair<T>(x0, x1) : 0u;
        const uint32_t b1 = lane < 4 ? pack_pair<T>(x2, x3) : 0u;
#pragma unroll
        for (int dt = 0; dt < DT; ++dt)
          mma16816<T>(acc_o[dt], va[kk][dt], b0, b1);
      }
    }

    // O^T column 0: dims 16dt + r (c0) and 16dt + 8 + r (c2) in lanes c == 0.
    // Fully masked rows: l == 0 and O == 0, so 0 * inf = NaN as in the
    // reference.
    const float inv = 1.f / l;
    if (c == 0) {
#pragma unroll
      for (int dt = 0; dt < DT; ++dt) {
        obuf[16 * dt + r] = acc_o[dt][0] * inv;
        obuf[16 * dt + 8 + r] = acc_o[dt][2] * inv;
      }
    }
    __syncwarp();
    if (lane < D / 8) {
      const float4 o0 = *reinterpret_cast<const float4*>(obuf + 8 * lane);
      const float4 o1 = *reinterpret_cast<const float4*>(obuf + 8 * lane + 4);
      uint4 u;
      u.x = pack_pair<T>(o0.x, o0.y);
      u.y = pack_pair<T>(o0.z, o0.w);
      u.z = pack_pair<T>(o1.x, o1.y);
      u.w = pack_pair<T>(o1.z, o1.w);
      *reinterpret_cast<uint4*>(gout + b * p.so[0] + h * p.so[1] +
                                8 * lane) = u;
    }
    __syncwarp();
  }
}

template <typename T, int D>
cudaError_t launch_t(const RbfProblem& p, cudaStream_t stream) {
  using Cfg = DmCfg<D>;
  if (!tensor_maps_available()) return cudaErrorNotSupported;
  CUtensorMap tk, tv;
  if (!make_tile_map(&tk, p.k, p.dtype, p.B, p.H, p.Nk, D, p.sk, kBoxRows) ||
      !make_tile_map(&tv, p.v, p.dtype, p.B, p.H, p.Nk, D, p.sv, kBoxRows))
    return cudaErrorInvalidValue;
  const size_t budget = 227 * 1024;
  int ns = static_cast<int>((budget - Cfg::block_bytes(0, kWarps)) /
                            (Cfg::STAGE + Cfg::QB + Cfg::META + 8));
  if (ns > 64) ns = 64;
  if (ns < kWarps + 2) return cudaErrorInvalidConfiguration;
  DmLaunch L;
  L.ns = ns;
  L.n_planes = static_cast<int>(p.B * p.H);
  L.H = static_cast<int>(p.H);
  L.nchunks = static_cast<int>((p.Nk + Cfg::KC - 1) / Cfg::KC);
  int64_t blocks = L.n_planes;
  const int64_t cap = device_sm_count();
  if (blocks > cap) blocks = cap;
  const size_t smem = Cfg::block_bytes(ns, kWarps);
  auto kern = rbf_decode_mma_kernel<T, D>;
  static std::atomic<int> configured[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  if (dev < 0 || dev >= 64 || !configured[dev].load()) {
    cudaError_t err = cudaFuncSetAttribute(
        kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
        static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < 64) configured[dev].store(1);
  }
  return launch_pdl(kern, dim3(static_cast<unsigned>(blocks)),
                    dim3(kWarps * 32), smem, stream, tk, tv, p, L);
}

bool aligned16(const void* ptr) {
  return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0;
}

}  // namespace

bool decode_mma_supports(const RbfProblem& p) {
  if (p.Nq != 1 || p.Nk < 1) return false;
  if (p.dtype != VECTRA_BF16 && p.dtype != VECTRA_F16) return false;
  if (p.D != p.Dv || (p.D != 64 && p.D != 128)) return false;
  if (p.B * p.H > (int64_t(1) << 30) || p.Nk > (int64_t(1) << 30))
    return false;
  // q row: bulk copy (16-byte aligned); K, V: TMA (unit inner stride,
  // 16-byte strides); output: 16-byte stores.
  if (p.sq[3] != 1 || p.sk[3] != 1 || p.sv[3] != 1 || p.so[3] != 1)
    return false;
  if (!aligned16(p.q) || !aligned16(p.k) || !aligned16(p.v) ||
      !aligned16(p.out))
    return false;
  const int64_t sizes[3] = {p.B, p.H, p.Nk};
  for (int i = 0; i < 3; ++i)
    if (sizes[i] > 1 && (p.sk[i] < 0 || p.sv[i] < 0 || (p.sk[i] * 2) % 16 ||
                         (p.sv[i] * 2) % 16))
      return false;
  for (int i = 0; i < 2; ++i)
    if ((p.sq[i] * 2) % 16 || (p.so[i] * 2) % 16) return false;
  return true;
}

cudaError_t launch_decode_mma(const RbfProblem& p, cudaStream_t stream) {
  if (p.dtype == VECTRA_BF16)
    return p.D == 64 ? launch_t<__nv_bfloat16, 64>(p, stream)
                     : launch_t<__nv_bfloat16, 128>(p, stream);
  return p.D == 64 ? launch_t<__half, 64>(p, stream)
                   : launch_t<__half, 128>(p, stream);
}

}  // namespace vectra
