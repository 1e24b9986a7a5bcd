// rbf_common.cuh: problem description, element conversion and the PTX
// helpers (mbarriers, bulk copies, exp2) shared by the RBF-attention kernels.
//
// All kernels compute, per (b, h, i),
//   out = sum_j softmax_j(-g * ||q_i - k_j||^2 + bias_j) v_j,   g = scale[b,h]
// with a float32 online softmax in the exp2 domain (logits are multiplied by
// log2(e) once), following the reference kernel's loop
// (kernels/vectra_kernels/spatial_rbf_attention.py:120-174) and its
// `safe_max` rule for rows whose keys so far are all masked
// (kernels/vectra_kernels/reference.py:146-152).
#pragma once

#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "vectra_rbf.h"

namespace vectra {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegInf = -__builtin_huge_valf();

// Everything a kernel needs about one call, by value (kernel parameter).
// Strides are in elements; a broadcast dimension has stride 0.
struct RbfProblem {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  const void* scale;
  const void* bias;  // nullptr: no bias
  int32_t dtype;        // of q, k, v and out
  int32_t scale_dtype;
  int32_t bias_dtype;
  int32_t pad_;
  int64_t B, H, Nq, Nk, D, Dv;
  int64_t sq[4], sk[4], sv[4], so[4];
  int64_t ss[2];  // scale strides over (b, h)
  int64_t sb[3];  // bias strides over (b, h, key)
  unsigned int* err;  // device error word (see report_error)
};

// Device error word: kernels set bits here instead of trapping. It is one
// `__device__` word per device owned by capi.cu, whose address reaches the
// kernels through RbfProblem::err.
enum : unsigned {
  kErrWaitTimeout = 1u,  // an mbarrier wait ran past its iteration limit
  kErrTmemAlloc = 2u,    // TMEM allocation did not succeed
};

__device__ __forceinline__ void report_error(unsigned int* err,
                                             unsigned bits) {
  if (err) atomicOr(err, bits);
}

// ---------------------------------------------------------------------------
// Element conversion.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) {
  return x;
}
template <> __device__ __forceinline__ __half from_f32<__half>(float x) {
  return __float2half_rn(x);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Loads element `idx` of a scale/bias array of runtime dtype as float.
__device__ __forceinline__ float load_any(const void* p, int dtype,
                                          int64_t idx) {
  switch (dtype) {
    case VECTRA_F32:
      return __ldg(static_cast<const float*>(p) + idx);
    case VECTRA_F16:
      return __half2float(__ldg(static_cast<const __half*>(p) + idx));
    case VECTRA_BF16:
      return __bfloat162float(
          __ldg(static_cast<const __nv_bfloat16*>(p) + idx));
    default:
      return static_cast<float>(__ldg(static_cast<const double*>(p) + idx));
  }
}

__device__ __forceinline__ float load_scale(const RbfProblem& p, int64_t b,
                                            int64_t h) {
  return load_any(p.scale, p.scale_dtype, b * p.ss[0] + h * p.ss[1]);
}

__device__ __forceinline__ float load_bias(const RbfProblem& p, int64_t b,
                                           int64_t h, int64_t key) {
  return load_any(p.bias, p.bias_dtype,
                  b * p.sb[0] + h * p.sb[1] + key * p.sb[2]);
}

// The bits of a bias element, loaded without converting it, so that the
// load can stay in flight until the value is used: 32-bit elements as they
// are, 16-bit ones zero-extended; a float64 bias is converted to float32
// bits on the spot.
__device__ __forceinline__ uint32_t load_bias_bits(const RbfProblem& p,
                                                   int64_t b, int64_t h,
                                                   int64_t key) {
  const int64_t idx = b * p.sb[0] + h * p.sb[1] + key * p.sb[2];
  switch (p.bias_dtype) {
    case VECTRA_F32:
      return __ldg(static_cast<const unsigned int*>(p.bias) + idx);
    case VECTRA_F16:
    case VECTRA_BF16:
      return __ldg(static_cast<const unsigned short*>(p.bias) + idx);
    default:
      return __float_as_uint(
          static_cast<float>(__ldg(static_cast<const double*>(p.bias) + idx)));
  }
}

// The bits of a scale element, loaded like load_bias_bits (convert with
// bias_bits_to_f32 and the scale's dtype).
__device__ __forceinline__ uint32_t load_scale_bits(const RbfProblem& p,
                                                    int64_t b, int64_t h) {
  const int64_t idx = b * p.ss[0] + h * p.ss[1];
  switch (p.scale_dtype) {
    case VECTRA_F32:
      return __ldg(static_cast<const unsigned int*>(p.scale) + idx);
    case VECTRA_F16:
    case VECTRA_BF16:
      return __ldg(static_cast<const unsigned short*>(p.scale) + idx);
    default:
      return __float_as_uint(static_cast<float>(
          __ldg(static_cast<const double*>(p.scale) + idx)));
  }
}
// The float value of bits from load_bias_bits (or load_scale_bits).
__device__ __forceinline__ float bias_bits_to_f32(uint32_t w, int dtype) {
  switch (dtype) {
    case VECTRA_F16:
      return __half2float(__ushort_as_half(static_cast<unsigned short>(w)));
    case VECTRA_BF16:
      return __uint_as_float(w << 16);
    default:
      return __uint_as_float(w);
  }
}

// 2^x on the SFU (ex2.approx: relative error ~2^-22; 2^-inf = +0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// ---------------------------------------------------------------------------
// mbarrier and bulk-copy (TMA, untiled) helpers. Waits are bounded: past
// kWaitLimit polls they record kErrWaitTimeout and return false, so a lost
// transfer becomes a host-visible error instead of a hung GPU.
// ---------------------------------------------------------------------------
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar),
               "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(phase)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t phase,
                                          unsigned int* err) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, phase)) return true;
  report_error(err, kErrWaitTimeout);
  return false;
}

// try_wait that lets the hardware suspend the thread (up to `hint_ns`)
// until the phase completes, so waiting warps take no issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar,
                                                    uint32_t phase,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(phase), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait of at most kSleepWaitLimit suspended polls of 20 us each
// (about 2 s in all) before recording kErrWaitTimeout.
constexpr uint32_t kSleepWaitLimit = 100000;
__device__ __forceinline__ bool mbar_wait_sleep(uint32_t bar, uint32_t phase,
                                                unsigned int* err) {
  for (uint32_t i = 0; i < kSleepWaitLimit; ++i)
    if (mbar_try_wait_sleep(bar, phase, 20000)) return true;
  report_error(err, kErrWaitTimeout);
  return false;
}

// Release store / acquire load of a shared-memory word (CTA scope), for
// publishing "stage s now holds item i" between warps.
__device__ __forceinline__ void st_release_smem(int* ptr, int v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_addr(ptr)),
               "r"(v)
               : "memory");
}
__device__ __forceinline__ int ld_acquire_smem(const int* ptr) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];"
               : "=r"(v)
               : "r"(smem_addr(ptr))
               : "memory");
  return v;
}

// Waits (bounded, about 2 s) until *ptr == want, backing off between
// polls; false (error recorded) on timeout.
__device__ __forceinline__ bool wait_smem_equals(const int* ptr, int want,
                                                 unsigned int* err) {
  unsigned sleep_ns = 32;
  for (uint32_t i = 0; i < kSleepWaitLimit; ++i) {
    if (ld_acquire_smem(ptr) == want) return true;
    __nanosleep(sleep_ns);
    if (sleep_ns < 512) sleep_ns <<= 1;
  }
  report_error(err, kErrWaitTimeout);
  return false;
}

// Global -> shared bulk copy completing `bytes` of transaction on `bar`.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src,
                                         uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// L2 policy for data read exactly once (streamed keys and values).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;"
               : "=l"(policy));
  return policy;
}

// L2 policy with the default (normal) eviction priority.
__device__ __forceinline__ uint64_t l2_evict_normal_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;"
               : "=l"(policy));
  return policy;
}

// Programmatic dependent launch. A kernel launched with launch_pdl may
// start while the previous kernel in the stream is still running; it calls
// allow_dependents() early (the next such kernel may then be scheduled as
// SMs free up) and grid_dependency_wait() before its first global-memory
// access, which returns once every earlier kernel has completed and its
// writes are visible. So inputs produced, and buffers read, by the previous
// kernel are ordered exactly as with a plain launch; only the launch
// latency and the shared-memory set-up overlap. Without a programmatic
// dependency both instructions are no-ops.
__device__ __forceinline__ void allow_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

#ifndef VECTRA_PDL
#define VECTRA_PDL 1  // 0: plain launches (for comparison)
#endif
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                       size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = VECTRA_PDL ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Kernel launchers (one per translation unit). Each returns a cudaError_t.
cudaError_t launch_generic(const RbfProblem& p, cudaStream_t stream);
cudaError_t launch_decode(const RbfProblem& p, cudaStream_t stream);
// True when the decode kernel has an instantiation and the layout it needs.
bool decode_supports(const RbfProblem& p);
cudaError_t launch_tc(const RbfProblem& p, cudaStream_t stream);
bool tc_supports(const RbfProblem& p);
cudaError_t launch_small(const RbfProblem& p, cudaStream_t stream);
bool small_supports(const RbfProblem& p);
cudaError_t launch_small_tc(const RbfProblem& p, cudaStream_t stream);
bool small_tc_supports(const RbfProblem& p);

// TMA tensor maps (tma_maps.cu). A [B, H, N, D] bf16/f16 view with element
// strides s (s[3] == 1) as a 4-D map with a box of `box_cols` columns by
// `box_rows` rows, swizzled over the box's row (box_cols 64: 128 bytes,
// SWIZZLE_128B; 32: SWIZZLE_64B; 16: SWIZZLE_32B); rows past N and columns
// past D read as zeros.
bool tensor_maps_available();
bool make_tile_map(CUtensorMap* map, const void* base, int dtype, int64_t B,
                   int64_t H, int64_t N, int64_t D, const int64_t* s,
                   int box_rows, int box_cols = 64);

// Streaming-multiprocessor count of the current device (cached).
int device_sm_count();

// Device address of the library's error word on the current device (cached;
// null when it cannot be looked up). Kernels set kErr* bits there;
// vectra_rbf_check_device_errors reads and clears it.
unsigned int* device_error_ptr();

}  // namespace vectra
