// rbf_cpu.cpp: the CPU implementation of vectra::rbf_attention.
//
// The reference operator's default implementation runs on CPU tensors
// (kernels/vectra_kernels/custom_ops.py:52-72 ->
// reference.matmul_rbf_attention, reference.py:79-99): compiled graphs that
// the compile pass rewrote also run on CPU, and the reference's compiler and
// model test suites rely on that. This is that implementation for this
// library: CPU tensors dispatch here (by device, as the reference's
// registration does), CUDA tensors reach the sm_100a kernels and never come
// here.
//
// Semantics follow the reference's CPU formulation:
//   out[b,h,i,:] = sum_j softmax_j(-scale[b,h] * ||q_i - k_j||^2
//                                   + bias[b,h,i,j]) * v[b,h,j,:]
// with float32 arithmetic whatever the input dtype, the result in v's dtype,
// scale broadcast to [B, H, 1, 1] and key_bias broadcast to [B, H, Nq, Nk]
// (any broadcastable shape, like the reference's `logits + key_bias`; the
// CUDA path needs it constant across queries), a row whose logits are all
// -inf becomes NaN (as softmax makes it), and Nk = 0 gives zeros (an empty
// weighted sum). Distances are formed directly, sum_d (q_d - k_d)^2, which
// is never negative, so the reference's clamp of its expanded form is not
// needed.
//
// Parallel over (b, h) planes with ATen's thread pool.
#include <ATen/ATen.h>
#include <ATen/Parallel.h>

#include <cmath>
#include <limits>
#include <optional>
#include <vector>

namespace vectra_cpu {

namespace {

at::Tensor as_float(const at::Tensor& t) {
  TORCH_CHECK_VALUE(at::isFloatingType(t.scalar_type()),
                    "vectra::rbf_attention: expected floating-point "
                    "tensors, got ",
                    t.scalar_type());
  return t.to(at::kCPU, at::kFloat);
}

// [B, H, 1, 1]-broadcast view of the scale (element strides, 0 where
// broadcast).
at::Tensor broadcast_scale(const at::Tensor& scale, int64_t b, int64_t h) {
  at::Tensor s = as_float(scale);
  TORCH_CHECK_VALUE(s.dim() <= 4,
                    "scale must be broadcastable to [B, H, 1, 1]");
  while (s.dim() < 4) s = s.unsqueeze(0);
  TORCH_CHECK_VALUE(s.size(2) == 1 && s.size(3) == 1 &&
                        (s.size(0) == 1 || s.size(0) == b) &&
                        (s.size(1) == 1 || s.size(1) == h),
                    "scale must be broadcastable to [B, H, 1, 1]");
  return s.expand({b, h, 1, 1});
}

at::Tensor broadcast_bias(const at::Tensor& bias, int64_t b, int64_t h,
                          int64_t nq, int64_t nk) {
  at::Tensor t = as_float(bias);
  TORCH_CHECK_VALUE(t.dim() <= 4,
                    "key_bias must be broadcastable to [B, H, Nq, Nk]");
  while (t.dim() < 4) t = t.unsqueeze(0);
  const int64_t want[4] = {b, h, nq, nk};
  for (int i = 0; i < 4; ++i)
    TORCH_CHECK_VALUE(t.size(i) == 1 || t.size(i) == want[i],
                      "key_bias of shape ", bias.sizes(),
                      " is not broadcastable to [B, H, Nq, Nk]");
  return t.expand({b, h, nq, nk});
}

}  // namespace

at::Tensor rbf_attention_cpu(const at::Tensor& q, const at::Tensor& k,
                             const at::Tensor& v, const at::Tensor& scale,
                             const std::optional<at::Tensor>& key_bias,
                             at::IntArrayRef out_sizes,
                             at::IntArrayRef out_strides) {
  TORCH_CHECK_VALUE(q.dim() == 4 && k.dim() == 4 && v.dim() == 4,
                    "q, k and v must be rank 4 ([B, H, N, D])");
  const int64_t B = q.size(0), H = q.size(1), NQ = q.size(2), D = q.size(3);
  const int64_t NK = k.size(2), DV = v.size(3);
  TORCH_CHECK_VALUE(k.size(0) == B && k.size(1) == H && k.size(3) == D &&
                        v.size(0) == B && v.size(1) == H && v.size(2) == NK,
                    "q, k and v shapes do not agree: q ", q.sizes(), ", k ",
                    k.sizes(), ", v ", v.sizes());
  const at::Tensor qf = as_float(q).contiguous();
  const at::Tensor kf = as_float(k).contiguous();
  const at::Tensor vf = as_float(v).contiguous();
  const at::Tensor s = broadcast_scale(scale, B, H);
  std::optional<at::Tensor> bias;
  if (key_bias.has_value() && key_bias->defined())
    bias = broadcast_bias(*key_bias, B, H, NQ, NK);

  at::Tensor out32 = at::empty({B, H, NQ, DV}, qf.options());
  if (out32.numel() > 0) {
    const float* qp = qf.data_ptr<float>();
    const float* kp = kf.data_ptr<float>();
    const float* vp = vf.data_ptr<float>();
    const float* sp = s.data_ptr<float>();
    const int64_t ss0 = s.stride(0), ss1 = s.stride(1);
    const float* bp = bias ? bias->data_ptr<float>() : nullptr;
    int64_t bs[4] = {0, 0, 0, 0};
    if (bias)
      for (int i = 0; i < 4; ++i) bs[i] = bias->stride(i);
    float* op = out32.data_ptr<float>();
    const float kNaN = std::numeric_limits<float>::quiet_NaN();
    const float kNegInf = -std::numeric_limits<float>::infinity();
    at::parallel_for(0, B * H, 1, [&](int64_t begin, int64_t end) {
      std::vector<float> logit(size_t(NK > 0 ? NK : 1));
      std::vector<float> acc(size_t(DV > 0 ? DV : 1));
      for (int64_t plane = begin; plane < end; ++plane) {
        const int64_t b = plane / H, h = plane % H;
        const float gamma = sp[b * ss0 + h * ss1];
        const float* kq = kp + plane * NK * D;
        const float* vq = vp + plane * NK * DV;
        for (int64_t i = 0; i < NQ; ++i) {
          const float* qi = qp + (plane * NQ + i) * D;
          float* oi = op + (plane * NQ + i) * DV;
          if (NK == 0) {
            for (int64_t e = 0; e < DV; ++e) oi[e] = 0.f;
            continue;
          }
          float mx = kNegInf;
          for (int64_t j = 0; j < NK; ++j) {
            const float* kj = kq + j * D;
            float d2 = 0.f;
            for (int64_t d = 0; d < D; ++d) {
              const float diff = qi[d] - kj[d];
              d2 += diff * diff;
            }
            float l = -gamma * d2;
            if (bp != nullptr)
              l += bp[b * bs[0] + h * bs[1] + i * bs[2] + j * bs[3]];
            logit[size_t(j)] = l;
            mx = (l > mx || std::isnan(l)) ? l : mx;
          }
          if (std::isnan(mx) || mx == kNegInf ||
              mx == std::numeric_limits<float>::infinity()) {
            // All keys masked (0 / 0), a NaN logit, or an infinite one
            // (inf - inf): softmax gives NaN for the whole row.
            for (int64_t e = 0; e < DV; ++e) oi[e] = kNaN;
            continue;
          }
          for (int64_t e = 0; e < DV; ++e) acc[size_t(e)] = 0.f;
          float sum = 0.f;
          for (int64_t j = 0; j < NK; ++j) {
            const float p = std::exp(logit[size_t(j)] - mx);
            sum += p;
            const float* vj = vq + j * DV;
            for (int64_t e = 0; e < DV; ++e) acc[size_t(e)] += p * vj[e];
          }
          const float inv = 1.f / sum;
          for (int64_t e = 0; e < DV; ++e) oi[e] = acc[size_t(e)] * inv;
        }
      }
    });
  }
  at::Tensor out = at::empty_strided(out_sizes, out_strides,
                                     v.options().device(at::kCPU));
  out.copy_(out32);
  return out;
}

}  // namespace vectra_cpu
