// torch_ext.cpp: registers the CUDA kernel of vectra::rbf_attention.
//
// The schema is the reference's, unchanged:
//   vectra::rbf_attention(Tensor q, Tensor k, Tensor v, Tensor scale,
//                         Tensor? key_bias=None) -> Tensor
// (inferred by torch.library.custom_op at
// kernels/vectra_kernels/custom_ops.py:52-72). The CUDA implementation
// replaces _rbf_attention_cuda (custom_ops.py:75-85): it validates, reads
// strides, allocates the output and calls the C ABI of libvectra_rbf.so on
// the current stream. CPU tensors dispatch to this library's CPU
// implementation (rbf_cpu.cpp), the counterpart of the reference's default
// implementation; CUDA tensors always reach the CUDA kernels and never fall
// back to the CPU. The fake (meta) implementation lives in
// vectra_b200/custom_ops.py.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <optional>
#include <vector>

#include "vectra_rbf.h"

namespace vectra_cpu {
at::Tensor rbf_attention_cpu(const at::Tensor& q, const at::Tensor& k,
                             const at::Tensor& v, const at::Tensor& scale,
                             const std::optional<at::Tensor>& key_bias,
                             at::IntArrayRef out_sizes,
                             at::IntArrayRef out_strides);
}  // namespace vectra_cpu

namespace {

int32_t io_dtype(at::ScalarType t) {
  switch (t) {
    case at::kFloat:
      return VECTRA_F32;
    case at::kHalf:
      return VECTRA_F16;
    case at::kBFloat16:
      return VECTRA_BF16;
    case at::kDouble:
      return VECTRA_F64;
    default:
      return -1;
  }
}

vectra_tensor describe(const at::Tensor& t) {
  vectra_tensor d{};
  d.data = t.data_ptr();
  d.dtype = io_dtype(t.scalar_type());
  d.ndim = static_cast<int32_t>(t.dim());
  for (int64_t i = 0; i < t.dim(); ++i) {
    d.size[i] = t.size(i);
    d.stride[i] = t.stride(i);
  }
  return d;
}

// Scale and bias are small: bring them to q's device and a float dtype
// when they are not there already (the reference casts them to float32 on
// the device on every call, spatial_rbf_attention.py:208-213,221; here
// that copy only happens for unusual inputs).
at::Tensor side_input(const at::Tensor& t, const at::Tensor& q) {
  at::Tensor out = t;
  if (out.device() != q.device()) out = out.to(q.device());
  if (io_dtype(out.scalar_type()) < 0) out = out.to(at::kFloat);
  return out;
}

[[noreturn]] void raise_status(int status) {
  const char* msg = vectra_rbf_strerror(status);
  switch (status) {
    case VECTRA_ERR_UNSUPPORTED:
      TORCH_CHECK_NOT_IMPLEMENTED(false, "vectra::rbf_attention: ", msg);
    case VECTRA_ERR_CUDA:
    case VECTRA_ERR_DEVICE:
      TORCH_CHECK(false, "vectra::rbf_attention: ", msg);
    default:
      TORCH_CHECK_VALUE(false, msg);
  }
  TORCH_CHECK(false, "unreachable");
}

// The output follows q's order of heads and tokens: when q's tokens are
// outer to its heads (a head-split view of a [B, N, H * D] projection), out
// is a head-transposed view of [B, Nq, H, Dv] memory, as PyTorch's
// attention kernels return, so out.transpose(1, 2).reshape(B, Nq, H * Dv)
// needs no copy; otherwise out is contiguous [B, H, Nq, Dv]. The fake
// implementation (vectra_b200/custom_ops.py) applies the same rule.
bool tokens_outer(const at::Tensor& q) {
  return q.size(1) > 1 && q.size(2) > 1 && q.stride(2) > q.stride(1);
}

std::vector<int64_t> output_strides(const at::Tensor& q, int64_t dv) {
  const int64_t h = q.size(1), n = q.size(2);
  if (tokens_outer(q)) return {n * h * dv, dv, h * dv, 1};
  return {h * n * dv, n * dv, dv, 1};
}

at::Tensor empty_output(const at::Tensor& q, const at::Tensor& v) {
  const int64_t dv = v.size(3);
  return at::empty_strided({q.size(0), q.size(1), q.size(2), dv},
                           output_strides(q, dv), v.options());
}

// Validates, allocates the output and launches through the C ABI.
at::Tensor run(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
               const at::Tensor& scale,
               const std::optional<at::Tensor>& key_bias, uint32_t flags) {
  TORCH_CHECK_VALUE(q.dim() == 4 && k.dim() == 4 && v.dim() == 4,
                    "q, k and v must be rank 4 ([B, H, N, D])");
  TORCH_CHECK_VALUE(q.is_cuda() && k.device() == q.device() &&
                        v.device() == q.device(),
                    "q, k and v must be on one CUDA device");
  TORCH_CHECK_VALUE(
      q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type(),
      "q, k and v must share a dtype");
  c10::cuda::CUDAGuard guard(q.device());
  const at::Tensor s = side_input(scale, q);
  std::optional<at::Tensor> bias;
  if (key_bias.has_value() && key_bias->defined())
    bias = side_input(*key_bias, q);

  at::Tensor out = empty_output(q, v);
  vectra_rbf_args a{};
  a.q = describe(q);
  a.k = describe(k);
  a.v = describe(v);
  a.scale = describe(s);
  if (bias) a.key_bias = describe(*bias);
  a.out = out.data_ptr();
  for (int i = 0; i < 4; ++i) a.out_stride[i] = out.stride(i);
  a.flags = flags;
  const int status = vectra_rbf_attention_forward(
      &a, at::cuda::getCurrentCUDAStream(q.device().index()).stream());
  if (status != VECTRA_OK) raise_status(status);
  return out;
}

at::Tensor rbf_attention_cuda(const at::Tensor& q, const at::Tensor& k,
                              const at::Tensor& v, const at::Tensor& scale,
                              const std::optional<at::Tensor>& key_bias) {
  return run(q, k, v, scale, key_bias, 0);
}

// vectra_b200::rbf_attention_with_flags: the same operator with an explicit
// kernel choice (VECTRA_FLAG_*), for tests and benchmarks that pin a kernel.
at::Tensor rbf_attention_flags_cuda(const at::Tensor& q, const at::Tensor& k,
                                    const at::Tensor& v,
                                    const at::Tensor& scale,
                                    const std::optional<at::Tensor>& key_bias,
                                    int64_t flags) {
  return run(q, k, v, scale, key_bias, static_cast<uint32_t>(flags));
}

// The CPU implementation: same output layout rule as the CUDA one.
at::Tensor rbf_attention_cpu_impl(const at::Tensor& q, const at::Tensor& k,
                                  const at::Tensor& v, const at::Tensor& scale,
                                  const std::optional<at::Tensor>& key_bias) {
  TORCH_CHECK_VALUE(q.dim() == 4 && k.dim() == 4 && v.dim() == 4,
                    "q, k and v must be rank 4 ([B, H, N, D])");
  const int64_t dv = v.size(3);
  return vectra_cpu::rbf_attention_cpu(
      q, k, v, scale, key_bias, {q.size(0), q.size(1), q.size(2), dv},
      output_strides(q, dv));
}

}  // namespace

TORCH_LIBRARY(vectra, m) {
  m.def(
      "rbf_attention(Tensor q, Tensor k, Tensor v, Tensor scale, "
      "Tensor? key_bias=None) -> Tensor");
}

TORCH_LIBRARY_IMPL(vectra, CUDA, m) {
  m.impl("rbf_attention", &rbf_attention_cuda);
}

TORCH_LIBRARY_IMPL(vectra, CPU, m) {
  m.impl("rbf_attention", &rbf_attention_cpu_impl);
}

TORCH_LIBRARY(vectra_b200, m) {
  m.def(
      "rbf_attention_with_flags(Tensor q, Tensor k, Tensor v, Tensor scale, "
      "Tensor? key_bias, int flags) -> Tensor");
}

TORCH_LIBRARY_IMPL(vectra_b200, CUDA, m) {
  m.impl("rbf_attention_with_flags", &rbf_attention_flags_cuda);
}
