/*
 * vectra_rbf.h: C ABI of the B200 RBF-attention library (libvectra_rbf.so).
 *
 * Computes, for every batch row b, head h and query i,
 *
 *   out[b,h,i,:] = sum_j softmax_j(-scale[b,h] * ||q[b,h,i,:] - k[b,h,j,:]||^2
 *                                  + key_bias[b,h,j]) * v[b,h,j,:]
 *
 * the operator `torch.ops.vectra.rbf_attention(q, k, v, scale, key_bias)`
 * of the reference (kernels/vectra_kernels/custom_ops.py:52-72), on CUDA
 * tensors, with hand-written sm_100a kernels.
 *
 * Conventions
 *  - Plain C: pointers, sizes and element strides. No allocation happens
 *    inside the library; the caller owns every buffer, including `out`.
 *  - Every call is asynchronous on the given CUDA stream (`cudaStream_t`
 *    passed as void*; NULL is the legacy default stream) and never
 *    synchronises, except vectra_rbf_check_device_errors.
 *  - Functions return VECTRA_OK (0) or a negative status; they never abort
 *    the process. vectra_rbf_strerror turns a status into a message.
 *  - Thread-safe and re-entrant across host threads and devices: the only
 *    global state is a per-device error word and a launch counter.
 */
#ifndef VECTRA_RBF_H_
#define VECTRA_RBF_H_

#include <stdint.h>

/* Only the functions below are exported from libvectra_rbf.so; the library
 * is built with hidden visibility for everything else. */
#ifndef VECTRA_API
#define VECTRA_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of tensors crossing the ABI. q, k and v share one of
 * F32 / F16 / BF16 (the reference accepts exactly these,
 * compiler/vectra_compiler/replacement.py:42); scale and key_bias may use
 * any of the four (the reference casts them to float32,
 * kernels/vectra_kernels/spatial_rbf_attention.py:208-213,221). */
typedef enum {
  VECTRA_F32 = 0,
  VECTRA_F16 = 1,
  VECTRA_BF16 = 2,
  VECTRA_F64 = 3
} vectra_dtype;

/* Status codes. */
enum {
  VECTRA_OK = 0,
  VECTRA_ERR_NULL = -1,         /* a required pointer is NULL */
  VECTRA_ERR_RANK = -2,         /* q, k or v is not rank 4; scale/bias rank > 4 */
  VECTRA_ERR_SHAPE = -3,        /* q, k, v sizes disagree */
  VECTRA_ERR_DTYPE = -4,        /* unsupported or mismatched element type */
  VECTRA_ERR_SCALE_SHAPE = -5,  /* scale does not broadcast to [B,H,1,1] */
  VECTRA_ERR_BIAS_SHAPE = -6,   /* key_bias does not broadcast to [B,1|H,1,Nk] */
  VECTRA_ERR_BIAS_QUERY = -7,   /* key_bias.shape[-2] != 1 ("key_bias must be
                                   constant across queries",
                                   spatial_rbf_attention.py:224-225) */
  VECTRA_ERR_UNSUPPORTED = -8,  /* head width beyond the kernels' limit (512) */
  VECTRA_ERR_CUDA = -9,         /* a CUDA runtime call failed */
  VECTRA_ERR_DEVICE = -10,      /* a kernel reported a bounded-wait timeout */
  VECTRA_ERR_FORCED = -11       /* the forced kernel cannot run this problem */
};

/* A strided view of up to 4 dimensions. Sizes and strides are in elements;
 * a stride of 0 broadcasts. Tensors of rank < 4 are read as left-padded
 * with size-1 dimensions (the reference's rule for scale and key_bias). */
typedef struct {
  const void* data;
  int32_t dtype;     /* vectra_dtype */
  int32_t ndim;      /* 0..4 */
  int64_t size[4];
  int64_t stride[4];
} vectra_tensor;

/* Kernel selection flags (0 = automatic; bit 0x8 is retired and, like any
 * other unknown bit, makes the call fail with VECTRA_ERR_FORCED). */
#define VECTRA_FLAG_FORCE_GENERIC 0x1u /* the any-shape tiled kernel */
#define VECTRA_FLAG_FORCE_DECODE  0x2u /* the Nq == 1 streaming kernel */
#define VECTRA_FLAG_FORCE_TC      0x4u /* the tcgen05/TMEM tensor-core kernel */
#define VECTRA_FLAG_FORCE_SMALL   0x10u /* the one-tile-per-plane kernel */
#define VECTRA_FLAG_FORCE_SMALL_TC 0x20u /* its tcgen05/TMEM form */

/* Kernels (vectra_rbf_select_kernel's result). */
enum {
  VECTRA_KERNEL_NONE = 0,     /* nothing to launch (an empty problem) */
  VECTRA_KERNEL_GENERIC = 1,  /* rbf_generic: any shape, stride and dtype */
  VECTRA_KERNEL_DECODE = 2,   /* rbf_decode: Nq == 1, bulk-copy streaming */
  VECTRA_KERNEL_TC = 3,       /* rbf_tc: tcgen05 + TMEM, long sequences */
  /* 4 is retired (an Nq == 1 mma.sync kernel, never chosen automatically) */
  VECTRA_KERNEL_SMALL = 5,      /* rbf_small: Nk <= 128, mma.sync tiles */
  VECTRA_KERNEL_SMALL_TC = 6    /* rbf_small_tc: Nq <= 96, Nk <= 128 - D,
                                   tcgen05 + TMEM; only when forced */
};

/* Arguments of one forward call.
 *  q [B,H,Nq,D], k [B,H,Nk,D], v [B,H,Nk,Dv]: same dtype, any strides.
 *  scale: broadcastable to [B,H,1,1]; zero and negative values are legal.
 *  key_bias: key_bias.data == NULL means no bias; otherwise broadcastable
 *    to [B,1|H,1,Nk] (0 / -inf for padded keys).
 *  out: [B,H,Nq,Dv] in v's dtype, with element strides out_stride.
 *  Rows whose keys are all masked come out NaN, as in the reference. */
typedef struct {
  vectra_tensor q, k, v, scale, key_bias;
  void* out;
  int64_t out_stride[4];
  uint32_t flags;
} vectra_rbf_args;

/* Launches RBF attention on `stream`.
 * Replaces rbf_attention_forward (kernels/vectra_kernels/
 * spatial_rbf_attention.py:177-281) and the CUDA registration
 * _rbf_attention_cuda (kernels/vectra_kernels/custom_ops.py:75-85). */
VECTRA_API int vectra_rbf_attention_forward(const vectra_rbf_args* args, void* stream);

/* Validates `args` and returns the VECTRA_KERNEL_* that forward would
 * launch, or a negative status (the same checks forward makes). Replaces
 * the tile heuristic tile_configs.select (kernels/vectra_kernels/
 * tile_configs.py:114-133). */
VECTRA_API int vectra_rbf_select_kernel(const vectra_rbf_args* args);

/* Name of a VECTRA_KERNEL_* value ("none", "generic", "decode", "tc",
 * "small", "small_tc"; "invalid" for any other value). */
VECTRA_API const char* vectra_rbf_kernel_name(int kernel);

/* Message for a status code. */
VECTRA_API const char* vectra_rbf_strerror(int status);

/* Synchronises `stream`, then reads and clears the current device's error
 * word, which kernels set instead of trapping when a bounded wait runs out.
 * Returns VECTRA_OK, VECTRA_ERR_DEVICE or VECTRA_ERR_CUDA. */
VECTRA_API int vectra_rbf_check_device_errors(void* stream);

/* Test hook for the failure path (no counterpart in the reference): launches,
 * on `stream`, a one-thread kernel whose bounded mbarrier wait can never
 * complete. After about 2 s the wait gives up, records the timeout in the
 * device error word and the kernel returns, as every kernel of the library
 * does when a wait runs out; vectra_rbf_check_device_errors then reports
 * VECTRA_ERR_DEVICE once and the context stays usable. Returns VECTRA_OK or
 * VECTRA_ERR_CUDA (launch failed). */
VECTRA_API int vectra_rbf_selftest_wait_timeout(void* stream);

/* Kernels launched by this library in this process (all devices). Tests
 * and the benchmark use it to prove the CUDA path ran. */
VECTRA_API uint64_t vectra_rbf_launch_count(void);

/* Build description: version, target architecture, compiler. */
VECTRA_API const char* vectra_rbf_build_info(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* VECTRA_RBF_H_ */
