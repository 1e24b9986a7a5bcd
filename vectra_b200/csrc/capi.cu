// capi.cu: the C ABI of libvectra_rbf.so (declared in include/vectra_rbf.h).
//
// Validates a call the way the reference's host wrapper does
// (kernels/vectra_kernels/spatial_rbf_attention.py:177-281): q, k, v rank 4
// with one dtype; scale broadcast to [B,H,1,1] in any float dtype; key_bias
// left-padded to rank 4, constant across queries, broadcast over batch and
// heads. Unlike the reference it makes no device copies of scale or bias
// (kernels read them in their own dtype through broadcast strides), computes
// no separate norm pass, and picks the kernel for the shape (select()).
#include <atomic>
#include <cstdio>
#include <mutex>

#include "rbf_common.cuh"

namespace vectra {

__device__ unsigned int g_vectra_device_error = 0;

namespace {

std::atomic<uint64_t> g_launches{0};

// Self-test of the kernels' failure path: waits on an mbarrier that nothing
// ever completes, through the same bounded wait the kernels use
// (mbar_wait_sleep, about 2 s), which records kErrWaitTimeout in the device
// error word and returns false. One thread, nothing else to wait for.
__global__ void wait_timeout_selftest_kernel(unsigned int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(smem_addr(&bar), 1);
  fence_barrier_init();
  mbar_wait_sleep(smem_addr(&bar), 0, err);  // no arrive: runs out
}

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<unsigned int*> g_err_ptr[kMaxDevices];

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

bool is_io_dtype(int32_t d) {
  return d == VECTRA_F32 || d == VECTRA_F16 || d == VECTRA_BF16;
}

bool is_any_dtype(int32_t d) { return is_io_dtype(d) || d == VECTRA_F64; }

// Size and stride of dimension i (0..3) of t, left-padded to rank 4.
int64_t padded_size(const vectra_tensor& t, int i) {
  const int off = 4 - t.ndim;
  return i < off ? 1 : t.size[i - off];
}
int64_t padded_stride(const vectra_tensor& t, int i) {
  const int off = 4 - t.ndim;
  return i < off ? 0 : t.stride[i - off];
}

// Fills `p` from `a`; returns VECTRA_OK or a status.
int build_problem(const vectra_rbf_args* a, RbfProblem* p) {
  if (a == nullptr) return VECTRA_ERR_NULL;
  const vectra_tensor &q = a->q, &k = a->k, &v = a->v;
  if (q.ndim != 4 || k.ndim != 4 || v.ndim != 4) return VECTRA_ERR_RANK;
  if (!is_io_dtype(q.dtype) || k.dtype != q.dtype || v.dtype != q.dtype)
    return VECTRA_ERR_DTYPE;
  *p = RbfProblem{};
  p->B = q.size[0];
  p->H = q.size[1];
  p->Nq = q.size[2];
  p->D = q.size[3];
  p->Nk = k.size[2];
  p->Dv = v.size[3];
  for (int i = 0; i < 4; ++i)
    if (q.size[i] < 0 || k.size[i] < 0 || v.size[i] < 0)
      return VECTRA_ERR_SHAPE;
  if (k.size[0] != p->B || k.size[1] != p->H || k.size[3] != p->D ||
      v.size[0] != p->B || v.size[1] != p->H || v.size[2] != p->Nk)
    return VECTRA_ERR_SHAPE;
  for (int i = 0; i < 4; ++i) {
    p->sq[i] = q.stride[i];
    p->sk[i] = k.stride[i];
    p->sv[i] = v.stride[i];
    p->so[i] = a->out_stride[i];
  }
  p->dtype = q.dtype;
  p->q = q.data;
  p->k = k.data;
  p->v = v.data;
  p->out = a->out;

  // scale: broadcastable to [B, H, 1, 1] (reference.py:41-43).
  const vectra_tensor& s = a->scale;
  if (s.data == nullptr) return VECTRA_ERR_NULL;
  if (s.ndim < 0 || s.ndim > 4) return VECTRA_ERR_RANK;
  if (!is_any_dtype(s.dtype)) return VECTRA_ERR_DTYPE;
  const int64_t s0 = padded_size(s, 0), s1 = padded_size(s, 1);
  if (padded_size(s, 2) != 1 || padded_size(s, 3) != 1 ||
      (s0 != 1 && s0 != p->B) || (s1 != 1 && s1 != p->H))
    return VECTRA_ERR_SCALE_SHAPE;
  p->scale = s.data;
  p->scale_dtype = s.dtype;
  p->ss[0] = s0 == 1 ? 0 : padded_stride(s, 0);
  p->ss[1] = s1 == 1 ? 0 : padded_stride(s, 1);

  // key_bias: optional, [B, 1|H, 1, Nk] (spatial_rbf_attention.py:220-234).
  const vectra_tensor& kb = a->key_bias;
  if (kb.data != nullptr) {
    if (kb.ndim < 0 || kb.ndim > 4) return VECTRA_ERR_RANK;
    if (!is_any_dtype(kb.dtype)) return VECTRA_ERR_DTYPE;
    if (padded_size(kb, 2) != 1) return VECTRA_ERR_BIAS_QUERY;
    const int64_t b0 = padded_size(kb, 0), b1 = padded_size(kb, 1),
                  b3 = padded_size(kb, 3);
    if ((b0 != 1 && b0 != p->B) || (b1 != 1 && b1 != p->H) ||
        (b3 != 1 && b3 != p->Nk))
      return VECTRA_ERR_BIAS_SHAPE;
    p->bias = kb.data;
    p->bias_dtype = kb.dtype;
    p->sb[0] = b0 == 1 ? 0 : padded_stride(kb, 0);
    p->sb[1] = b1 == 1 ? 0 : padded_stride(kb, 1);
    p->sb[2] = b3 == 1 ? 0 : padded_stride(kb, 3);
  }

  const bool empty = p->B == 0 || p->H == 0 || p->Nq == 0 || p->Dv == 0;
  if (!empty) {
    if (p->out == nullptr || p->q == nullptr) return VECTRA_ERR_NULL;
    if (p->Nk > 0 && (p->k == nullptr || p->v == nullptr))
      return VECTRA_ERR_NULL;
    if (p->D > 512 || p->Dv > 512) return VECTRA_ERR_UNSUPPORTED;
  }
  return VECTRA_OK;
}

int select(const RbfProblem& p, uint32_t flags) {
  constexpr uint32_t kKnownFlags = VECTRA_FLAG_FORCE_GENERIC |
                                   VECTRA_FLAG_FORCE_DECODE |
                                   VECTRA_FLAG_FORCE_TC |
                                   VECTRA_FLAG_FORCE_SMALL |
                                   VECTRA_FLAG_FORCE_SMALL_TC;
  if (flags & ~kKnownFlags) return VECTRA_ERR_FORCED;
  if (p.B == 0 || p.H == 0 || p.Nq == 0 || p.Dv == 0)
    return VECTRA_KERNEL_NONE;
  if (flags & VECTRA_FLAG_FORCE_GENERIC) return VECTRA_KERNEL_GENERIC;
  if (flags & VECTRA_FLAG_FORCE_DECODE)
    return decode_supports(p) ? VECTRA_KERNEL_DECODE : VECTRA_ERR_FORCED;
  if (flags & VECTRA_FLAG_FORCE_TC)
    return tc_supports(p) ? VECTRA_KERNEL_TC : VECTRA_ERR_FORCED;
  if (flags & VECTRA_FLAG_FORCE_SMALL)
    return small_supports(p) ? VECTRA_KERNEL_SMALL : VECTRA_ERR_FORCED;
  if (flags & VECTRA_FLAG_FORCE_SMALL_TC)
    return small_tc_supports(p) ? VECTRA_KERNEL_SMALL_TC : VECTRA_ERR_FORCED;
  // Nq == 1: the SIMT decode kernel (an mma.sync variant measured slower
  // on every serving shape tried and is not built).
  if (decode_supports(p)) return VECTRA_KERNEL_DECODE;
  if (tc_supports(p)) return VECTRA_KERNEL_TC;
  // rbf_small_tc (tcgen05) runs only when forced: on the compiled model's
  // sites it measured slower than rbf_small (48.1 against 45.7 us).
  if (small_supports(p)) return VECTRA_KERNEL_SMALL;
  return VECTRA_KERNEL_GENERIC;
}


}  // namespace

int device_sm_count() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  int n = g_sm_count[dev].load(std::memory_order_relaxed);
  if (n > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) !=
          cudaSuccess ||
      n <= 0)
    n = 148;
  g_sm_count[dev].store(n, std::memory_order_relaxed);
  return n;
}

}  // namespace vectra

using namespace vectra;

namespace vectra {

// Device address of the error word on the current device (cached).
unsigned int* device_error_ptr() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  unsigned int* ptr = g_err_ptr[dev].load(std::memory_order_acquire);
  if (ptr) return ptr;
  void* addr = nullptr;
  if (cudaGetSymbolAddress(&addr, g_vectra_device_error) != cudaSuccess)
    return nullptr;
  ptr = static_cast<unsigned int*>(addr);
  g_err_ptr[dev].store(ptr, std::memory_order_release);
  return ptr;
}

}  // namespace vectra

extern "C" {

int vectra_rbf_select_kernel(const vectra_rbf_args* args) {
  RbfProblem p;
  const int st = build_problem(args, &p);
  if (st != VECTRA_OK) return st;
  return select(p, args->flags);
}

int vectra_rbf_attention_forward(const vectra_rbf_args* args, void* stream) {
  RbfProblem p;
  int st = build_problem(args, &p);
  if (st != VECTRA_OK) return st;
  const int kernel = select(p, args->flags);
  if (kernel < 0) return kernel;
  if (kernel == VECTRA_KERNEL_NONE) return VECTRA_OK;
  p.err = device_error_ptr();
  if (p.err == nullptr) return VECTRA_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  switch (kernel) {
    case VECTRA_KERNEL_DECODE:
      err = launch_decode(p, s);
      break;
    case VECTRA_KERNEL_TC:
      err = launch_tc(p, s);
      break;
    case VECTRA_KERNEL_SMALL:
      err = launch_small(p, s);
      break;
    case VECTRA_KERNEL_SMALL_TC:
      err = launch_small_tc(p, s);
      break;
    default:
      err = launch_generic(p, s);
      break;
  }
  if (err != cudaSuccess) return VECTRA_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return VECTRA_OK;
}

const char* vectra_rbf_kernel_name(int kernel) {
  switch (kernel) {
    case VECTRA_KERNEL_NONE:
      return "none";
    case VECTRA_KERNEL_GENERIC:
      return "generic";
    case VECTRA_KERNEL_DECODE:
      return "decode";
    case VECTRA_KERNEL_TC:
      return "tc";
    case VECTRA_KERNEL_SMALL:
      return "small";
    case VECTRA_KERNEL_SMALL_TC:
      return "small_tc";
    default:
      return "invalid";
  }
}

const char* vectra_rbf_strerror(int status) {
  switch (status) {
    case VECTRA_OK:
      return "ok";
    case VECTRA_ERR_NULL:
      return "a required pointer is NULL";
    case VECTRA_ERR_RANK:
      return "q, k and v must be rank 4 ([B, H, N, D]); scale and key_bias "
             "at most rank 4";
    case VECTRA_ERR_SHAPE:
      return "q [B,H,Nq,D], k [B,H,Nk,D] and v [B,H,Nk,Dv] sizes disagree";
    case VECTRA_ERR_DTYPE:
      return "q, k and v must share one of float32, float16, bfloat16; scale "
             "and key_bias must be floating point";
    case VECTRA_ERR_SCALE_SHAPE:
      return "scale must be broadcastable to [B, H, 1, 1]";
    case VECTRA_ERR_BIAS_SHAPE:
      return "key_bias must be broadcastable to [B, 1|H, 1, Nk]";
    case VECTRA_ERR_BIAS_QUERY:
      return "key_bias must be constant across queries";
    case VECTRA_ERR_UNSUPPORTED:
      return "unsupported size: a head width above 512, a scan's k above "
             "256, or a scan larger than the static scan scratch";
    case VECTRA_ERR_CUDA:
      return "a CUDA runtime call failed";
    case VECTRA_ERR_DEVICE:
      return "a kernel reported a bounded-wait timeout";
    case VECTRA_ERR_FORCED:
      return "the forced kernel cannot run this problem";
    default:
      return "unknown status";
  }
}

int vectra_rbf_check_device_errors(void* stream) {
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) !=
      cudaSuccess)
    return VECTRA_ERR_CUDA;
  unsigned int word = 0;
  if (cudaMemcpyFromSymbol(&word, g_vectra_device_error, sizeof(word)) !=
      cudaSuccess)
    return VECTRA_ERR_CUDA;
  if (word == 0) return VECTRA_OK;
  const unsigned int zero = 0;
  if (cudaMemcpyToSymbol(g_vectra_device_error, &zero, sizeof(zero)) !=
      cudaSuccess)
    return VECTRA_ERR_CUDA;
  return VECTRA_ERR_DEVICE;
}

int vectra_rbf_selftest_wait_timeout(void* stream) {
  unsigned int* err = device_error_ptr();
  if (err == nullptr) return VECTRA_ERR_CUDA;
  wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      err);
  return cudaGetLastError() == cudaSuccess ? VECTRA_OK : VECTRA_ERR_CUDA;
}

uint64_t vectra_rbf_launch_count(void) {
  return g_launches.load(std::memory_order_relaxed);
}

const char* vectra_rbf_build_info(void) {
  return "vectra_b200 0.1.0; sm_100a; nvcc " VECTRA_NVCC_VERSION;
}

}  // extern "C"
