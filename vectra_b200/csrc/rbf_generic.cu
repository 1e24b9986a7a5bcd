// rbf_generic.cu: RBF attention for any shape, stride and dtype.
//
// One 128-thread block per (query tile of kBQ rows, plane (b, h)), looping
// over key tiles of kBK keys with an online softmax; Q, K, V tiles are
// staged in shared memory as float32 (rows padded by one word so that
// column-wise reads hit distinct banks). Distances are formed directly as
// sum_d (q_d - k_d)^2 in float32, the eager formulation
// (kernels/vectra_kernels/reference.py:54), which needs no clamp and keeps
// full precision for far-apart points. Element strides are arbitrary, so
// head-transposed views (kernels/tests/test_edges.py:103-114) need no copy.
//
// This kernel is the correctness backbone: every problem the specialised
// kernels decline (odd head widths up to 512, Nq > 1 off the tensor-core
// path, non-unit innermost strides, fp32 off the decode path) runs here.
// Its roofline is the L2/SIMT one, not HBM; it is not a headline path. The
// common widths (D == Dv in {16, 32, 64, 128}) run a compile-time-width
// version of the same algorithm (rbf_generic_fixed_kernel).
#include "rbf_common.cuh"

namespace vectra {
namespace {

constexpr int kBQ = 16;       // query rows per block
constexpr int kBK = 32;       // keys per tile
constexpr int kThreads = 128; // 16 rows x 8 threads

struct GenericSmem {
  static size_t bytes(int64_t D, int64_t Dv) {
    return sizeof(float) * (kBQ * (D + 1) + kBK * (D + 1) + kBK * Dv +
                            kBQ * (kBK + 1) + kBQ * Dv + kBK);
  }
};

template <typename T>
__global__ void __launch_bounds__(kThreads)
    rbf_generic_kernel(RbfProblem p, int64_t n_qtiles, int64_t n_blocks) {
  extern __shared__ float smem[];
  const int D = static_cast<int>(p.D);
  const int Dv = static_cast<int>(p.Dv);
  const int DP = D + 1;
  float* Qs = smem;               // [kBQ][DP]
  float* Ks = Qs + kBQ * DP;      // [kBK][DP]
  float* Vs = Ks + kBK * DP;      // [kBK][Dv]
  float* Ps = Vs + kBK * Dv;      // [kBQ][kBK + 1]
  float* As = Ps + kBQ * (kBK + 1);  // [kBQ][Dv]
  float* Bs = As + kBQ * Dv;      // [kBK]

  const int tid = threadIdx.x;
  const int r = tid >> 3;  // query row within the tile
  const int c0 = tid & 7;  // first key column / value column of this thread
  const T* __restrict__ q = static_cast<const T*>(p.q);
  const T* __restrict__ k = static_cast<const T*>(p.k);
  const T* __restrict__ v = static_cast<const T*>(p.v);
  T* __restrict__ out = static_cast<T*>(p.out);
  allow_dependents();
  grid_dependency_wait();  // before any global access

  for (int64_t blk = blockIdx.x; blk < n_blocks; blk += gridDim.x) {
    const int64_t plane = blk / n_qtiles;
    const int64_t q0 = (blk % n_qtiles) * kBQ;
    const int64_t b = plane / p.H, h = plane % p.H;
    const T* qb = q + b * p.sq[0] + h * p.sq[1];
    const T* kb = k + b * p.sk[0] + h * p.sk[1];
    const T* vb = v + b * p.sv[0] + h * p.sv[1];

    __syncthreads();  // the previous block's readers are done
    for (int idx = tid; idx < kBQ * D; idx += kThreads) {
      const int rr = idx / D, d = idx - rr * D;
      const int64_t qi = q0 + rr;
      Qs[rr * DP + d] =
          qi < p.Nq ? to_f32(qb[qi * p.sq[2] + d * p.sq[3]]) : 0.f;
    }
    for (int idx = tid; idx < kBQ * Dv; idx += kThreads) As[idx] = 0.f;
    // The coefficient in the exp2 domain: logit2 = -(g * log2 e) * dist.
    const float g2 = load_scale(p, b, h) * kLog2e;
    float m = kNegInf, l = 0.f;

    for (int64_t k0 = 0; k0 < p.Nk; k0 += kBK) {
      __syncthreads();  // previous tile fully consumed
      for (int idx = tid; idx < kBK * D; idx += kThreads) {
        const int cc = idx / D, d = idx - cc * D;
        const int64_t kj = k0 + cc;
        Ks[cc * DP + d] =
            kj < p.Nk ? to_f32(kb[kj * p.sk[2] + d * p.sk[3]]) : 0.f;
      }
      for (int idx = tid; idx < kBK * Dv; idx += kThreads) {
        const int cc = idx / Dv, d = idx - cc * Dv;
        const int64_t kj = k0 + cc;
        Vs[cc * Dv + d] =
            kj < p.Nk ? to_f32(vb[kj * p.sv[2] + d * p.sv[3]]) : 0.f;
      }
      if (tid < kBK) {
        const int64_t kj = k0 + tid;
        float bias = kNegInf;  // keys past the end are masked
        if (kj < p.Nk) bias = p.bias ? load_bias(p, b, h, kj) * kLog2e : 0.f;
        Bs[tid] = bias;
      }
      __syncthreads();

      // Scores for row r, keys c0 + 8 i.
      float s[kBK / 8];
      float tmax = kNegInf;
#pragma unroll
      for (int i = 0; i < kBK / 8; ++i) {
        const int cc = c0 + 8 * i;
        const float* qr = Qs + r * DP;
        const float* kr = Ks + cc * DP;
        float dist = 0.f;
        for (int d = 0; d < D; ++d) {
          const float diff = qr[d] - kr[d];
          dist = fmaf(diff, diff, dist);
        }
        // -inf bias stays -inf; keys past Nk carry a -inf bias.
        s[i] = fmaf(-g2, dist, Bs[cc]);
        tmax = fmaxf(tmax, s[i]);
      }
      // Row max and sum over the 8 threads of row r (adjacent lanes).
#pragma unroll
      for (int o = 1; o < 8; o <<= 1)
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float m_new = fmaxf(m, tmax);
      const float safe = (m_new == kNegInf) ? 0.f : m_new;
      const float alpha = fast_exp2(m - safe);
      float psum = 0.f;
#pragma unroll
      for (int i = 0; i < kBK / 8; ++i) {
        const float pr = fast_exp2(s[i] - safe);
        Ps[r * (kBK + 1) + c0 + 8 * i] = pr;
        psum += pr;
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1)
        psum += __shfl_xor_sync(0xffffffffu, psum, o);
      l = l * alpha + psum;
      m = m_new;
      __syncthreads();  // Ps complete

      // As[r][d] = alpha * As[r][d] + sum_c P[r][c] V[c][d].
      for (int d = c0; d < Dv; d += 8) {
        float acc = As[r * Dv + d] * alpha;
#pragma unroll 8
        for (int cc = 0; cc < kBK; ++cc)
          acc = fmaf(Ps[r * (kBK + 1) + cc], Vs[cc * Dv + d], acc);
        As[r * Dv + d] = acc;
      }
    }

    // out = acc / l. Fully masked rows: 0 / 0 = NaN, like the reference;
    // no keys at all (Nk == 0): zeros, like softmax(empty) @ v.
    const int64_t qi = q0 + r;
    if (qi < p.Nq) {
      const float inv = (p.Nk == 0) ? 0.f : 1.f / l;
      T* orow = out + b * p.so[0] + h * p.so[1] + qi * p.so[2];
      for (int d = c0; d < Dv; d += 8)
        orow[d * p.so[3]] = from_f32<T>(As[r * Dv + d] * inv);
    }
  }
}

// The same algorithm for D == Dv in {16, 32, 64, 128}, with the width known
// at compile time: distance loops unrolled over 16-byte shared-memory reads
// (rows padded by 4 floats keep them aligned and put the 8 key rows a warp
// reads on distinct bank groups), the output row accumulated in registers
// across key tiles, and the probabilities of a query row shared only by the
// 8 threads of that row (one warp), so two CTA barriers per key tile.
template <typename T, int D>
__global__ void __launch_bounds__(kThreads)
    rbf_generic_fixed_kernel(RbfProblem p, int64_t n_qtiles,
                             int64_t n_blocks) {
  static_assert(D % 8 == 0 && D <= 128, "width");
  constexpr int DP = D + 4;        // row pitch in floats
  constexpr int PP = kBK + 4;      // probability row pitch
  constexpr int CH = D / 4;        // float4 chunks per row
  constexpr int NV = D / 8;        // output columns per thread
  extern __shared__ __align__(16) float smem[];
  float* Qs = smem;                // [kBQ][DP]
  float* Ks = Qs + kBQ * DP;       // [kBK][DP]
  float* Vs = Ks + kBK * DP;       // [kBK][DP]
  float* Ps = Vs + kBK * DP;       // [kBQ][PP]
  float* Bs = Ps + kBQ * PP;       // [kBK]

  const int tid = threadIdx.x;
  const int r = tid >> 3;   // query row within the tile (8 threads per row)
  const int c0 = tid & 7;   // key c0 + 8 i, output column c0 + 8 m
  const T* __restrict__ q = static_cast<const T*>(p.q);
  const T* __restrict__ k = static_cast<const T*>(p.k);
  const T* __restrict__ v = static_cast<const T*>(p.v);
  T* __restrict__ out = static_cast<T*>(p.out);
  allow_dependents();
  grid_dependency_wait();  // before any global access

  for (int64_t blk = blockIdx.x; blk < n_blocks; blk += gridDim.x) {
    const int64_t plane = blk / n_qtiles;
    const int64_t q0 = (blk % n_qtiles) * kBQ;
    const int64_t b = plane / p.H, h = plane % p.H;
    const T* qb = q + b * p.sq[0] + h * p.sq[1];
    const T* kb = k + b * p.sk[0] + h * p.sk[1];
    const T* vb = v + b * p.sv[0] + h * p.sv[1];

    __syncthreads();  // the previous block's readers are done
    for (int idx = tid; idx < kBQ * D; idx += kThreads) {
      const int rr = idx / D, d = idx % D;
      const int64_t qi = q0 + rr;
      Qs[rr * DP + d] =
          qi < p.Nq ? to_f32(qb[qi * p.sq[2] + d * p.sq[3]]) : 0.f;
    }
    const float g2 = load_scale(p, b, h) * kLog2e;
    float m = kNegInf, l = 0.f;
    float acc[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) acc[j] = 0.f;

    for (int64_t k0 = 0; k0 < p.Nk; k0 += kBK) {
      __syncthreads();  // previous tile fully consumed (and Qs written)
      for (int idx = tid; idx < kBK * D; idx += kThreads) {
        const int cc = idx / D, d = idx % D;
        const int64_t kj = k0 + cc;
        const bool in = kj < p.Nk;
        Ks[cc * DP + d] = in ? to_f32(kb[kj * p.sk[2] + d * p.sk[3]]) : 0.f;
        Vs[cc * DP + d] = in ? to_f32(vb[kj * p.sv[2] + d * p.sv[3]]) : 0.f;
      }
      if (tid < kBK) {
        const int64_t kj = k0 + tid;
        float bias = kNegInf;  // keys past the end are masked
        if (kj < p.Nk) bias = p.bias ? load_bias(p, b, h, kj) * kLog2e : 0.f;
        Bs[tid] = bias;
      }
      __syncthreads();

      // Distances of row r to keys c0 + 8 i.
      float dist[kBK / 8];
#pragma unroll
      for (int i = 0; i < kBK / 8; ++i) dist[i] = 0.f;
#pragma unroll
      for (int ch = 0; ch < CH; ++ch) {
        const float4 qv = *reinterpret_cast<const float4*>(Qs + r * DP + 4 * ch);
#pragma unroll
        for (int i = 0; i < kBK / 8; ++i) {
          const float4 kv = *reinterpret_cast<const float4*>(
              Ks + (c0 + 8 * i) * DP + 4 * ch);
          const float dx = qv.x - kv.x, dy = qv.y - kv.y;
          const float dz = qv.z - kv.z, dw = qv.w - kv.w;
          dist[i] = fmaf(dx, dx, dist[i]);
          dist[i] = fmaf(dy, dy, dist[i]);
          dist[i] = fmaf(dz, dz, dist[i]);
          dist[i] = fmaf(dw, dw, dist[i]);
        }
      }
      float s[kBK / 8];
      float tmax = kNegInf;
#pragma unroll
      for (int i = 0; i < kBK / 8; ++i) {
        // -inf bias stays -inf; keys past Nk carry a -inf bias.
        s[i] = fmaf(-g2, dist[i], Bs[c0 + 8 * i]);
        tmax = fmaxf(tmax, s[i]);
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1)
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float m_new = fmaxf(m, tmax);
      const float safe = (m_new == kNegInf) ? 0.f : m_new;
      const float alpha = fast_exp2(m - safe);
      float psum = 0.f;
#pragma unroll
      for (int i = 0; i < kBK / 8; ++i) {
        const float pr = fast_exp2(s[i] - safe);
        Ps[r * PP + c0 + 8 * i] = pr;
        psum += pr;
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1)
        psum += __shfl_xor_sync(0xffffffffu, psum, o);
      l = l * alpha + psum;
      m = m_new;
      __syncwarp();  // row r's probabilities: written and read in this warp

      // acc[j] = alpha * acc[j] + sum_c P[r][c] V[c][c0 + 8 j].
#pragma unroll
      for (int j = 0; j < NV; ++j) acc[j] *= alpha;
#pragma unroll 8
      for (int cc = 0; cc < kBK; ++cc) {
        const float pr = Ps[r * PP + cc];
#pragma unroll
        for (int j = 0; j < NV; ++j)
          acc[j] = fmaf(pr, Vs[cc * DP + c0 + 8 * j], acc[j]);
      }
    }

    // out = acc / l. Fully masked rows: 0 / 0 = NaN, like the reference;
    // no keys at all (Nk == 0): zeros, like softmax(empty) @ v.
    const int64_t qi = q0 + r;
    if (qi < p.Nq) {
      const float inv = (p.Nk == 0) ? 0.f : 1.f / l;
      T* orow = out + b * p.so[0] + h * p.so[1] + qi * p.so[2];
#pragma unroll
      for (int j = 0; j < NV; ++j)
        orow[(c0 + 8 * j) * p.so[3]] = from_f32<T>(acc[j] * inv);
    }
  }
}

template <typename T, int D>
cudaError_t launch_fixed(const RbfProblem& p, cudaStream_t stream,
                         int64_t n_qtiles, int64_t n_blocks) {
  constexpr int DP = D + 4;
  const size_t smem =
      sizeof(float) * (kBQ * DP + 2 * kBK * DP + kBQ * (kBK + 4) + kBK);
  cudaError_t err = cudaFuncSetAttribute(
      rbf_generic_fixed_kernel<T, D>,
      cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
  const unsigned grid =
      static_cast<unsigned>(n_blocks < cap ? n_blocks : cap);
  return launch_pdl(rbf_generic_fixed_kernel<T, D>, dim3(grid),
                    dim3(kThreads), smem, stream, p, n_qtiles, n_blocks);
}

template <typename T>
cudaError_t launch_generic_t(const RbfProblem& p, cudaStream_t stream) {
  const int64_t n_qtiles = (p.Nq + kBQ - 1) / kBQ;
  const int64_t n_blocks = n_qtiles * p.B * p.H;
  if (n_blocks == 0) return cudaSuccess;
  if (p.D == p.Dv) {
    switch (p.D) {
      case 16:
        return launch_fixed<T, 16>(p, stream, n_qtiles, n_blocks);
      case 32:
        return launch_fixed<T, 32>(p, stream, n_qtiles, n_blocks);
      case 64:
        return launch_fixed<T, 64>(p, stream, n_qtiles, n_blocks);
      case 128:
        return launch_fixed<T, 128>(p, stream, n_qtiles, n_blocks);
      default:
        break;
    }
  }
  const size_t smem = GenericSmem::bytes(p.D, p.Dv);
  cudaError_t err = cudaFuncSetAttribute(
      rbf_generic_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
      static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  // Enough resident blocks to fill the GPU; the kernel strides over the rest.
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
  const unsigned grid =
      static_cast<unsigned>(n_blocks < cap ? n_blocks : cap);
  return launch_pdl(rbf_generic_kernel<T>, dim3(grid), dim3(kThreads), smem,
                    stream, p, n_qtiles, n_blocks);
}

}  // namespace

cudaError_t launch_generic(const RbfProblem& p, cudaStream_t stream) {
  switch (p.dtype) {
    case VECTRA_F32:
      return launch_generic_t<float>(p, stream);
    case VECTRA_F16:
      return launch_generic_t<__half>(p, stream);
    default:
      return launch_generic_t<__nv_bfloat16>(p, stream);
  }
}

}  // namespace vectra
