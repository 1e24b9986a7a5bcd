"""torch.ops.vectra.rbf_attention on B200: the reference operator, re-backed.

Mirrors the reference module kernels/vectra_kernels/custom_ops.py: the same
operator name (`OP_NAME`, :44), the same schema (:52-59), the same fake
implementation (:88-97), and a CUDA implementation (:75-85) that is now the
C++ binding in _vectra_rbf_torch.so calling hand-written sm_100a kernels
through libvectra_rbf.so. Differences from the reference, on purpose:

* There is no Triton path and no "CUDA without Triton -> CPU arithmetic"
  fallback (custom_ops.py:39-42,83-84): if the extension is missing,
  importing this module raises.
* CPU tensors run this library's CPU implementation (csrc/rbf_cpu.cpp, a
  C++ loop parallel over planes), the counterpart of the reference's
  default implementation (custom_ops.py:52-72 ->
  reference.matmul_rbf_attention): float32 arithmetic, result in v's
  dtype, key_bias broadcast to [B, H, Nq, Nk]. Dispatch is by device, as
  in the reference; CUDA tensors never reach it.
* The output's layout follows q (`output_strides`): when q's tokens are
  outer to its heads (q a head-split view of a [B, N, H * D] projection,
  as in the compiled model), the output is a head-transposed view of
  [B, Nq, H, Dv] memory, as PyTorch's own attention kernels return, so the
  model's `.transpose(1, 2).reshape(B, N, H * Dv)` is a view instead of a
  copy; otherwise it is contiguous, as the reference's is. Values are the
  same either way.

Typical usage (unchanged):

    out = torch.ops.vectra.rbf_attention(q, k, v, scale, key_bias)
"""

import torch

from vectra_b200 import _lib

OP_NAME = 'vectra::rbf_attention'

torch.ops.load_library(_lib.TORCH_EXT_PATH)


def output_strides(q, dv: int) -> tuple:
    """Strides of the operator's [B, H, Nq, Dv] output for query q: those of
    a head-transposed view of [B, Nq, H, Dv] memory when q's tokens are
    outer to its heads (H > 1, Nq > 1, q.stride(2) > q.stride(1)), else
    contiguous. The CUDA implementation allocates the same way
    (csrc/torch_ext.cpp)."""
    b, h, n = q.shape[0], q.shape[1], q.shape[2]
    if h > 1 and n > 1 and q.stride(2) > q.stride(1):
        return (n * h * dv, dv, h * dv, 1)
    return (h * n * dv, n * dv, dv, 1)


def _empty_output(q, v):
    dv = v.shape[-1]
    return q.new_empty_strided((*q.shape[:-1], dv), output_strides(q, dv),
                               dtype=v.dtype)


@torch.library.register_fake(OP_NAME)
def _rbf_attention_fake(q, k, v, scale, key_bias=None):
    del k, scale, key_bias  # Only the output's shape and layout matter here.
    return _empty_output(q, v)


@torch.library.register_fake('vectra_b200::rbf_attention_with_flags')
def _rbf_attention_with_flags_fake(q, k, v, scale, key_bias, flags):
    del k, scale, key_bias, flags
    return _empty_output(q, v)


def cuda_available() -> bool:
    """Whether the B200 kernels can run here (the reference's
    `triton_available`, custom_ops.py:47-49)."""
    return torch.cuda.is_available()


def rbf_attention(q, k, v, scale, key_bias=None) -> torch.Tensor:
    """Fused RBF attention: softmax(-scale * ||q - k||^2 + key_bias) @ v.

    Args:
      q: [B, H, Nq, D] (float32, float16 or bfloat16), any strides; CUDA
        tensors run the sm_100a kernels, CPU tensors the CPU implementation.
      k: [B, H, Nk, D], same dtype.
      v: [B, H, Nk, Dv], same dtype.
      scale: Broadcastable to [B, H, 1, 1]; the RBF coefficient
        1 / (2 sigma^2). Zero and negative values are legal.
      key_bias: Optional, broadcastable to [B, 1|H, 1, Nk]; 0 for real keys
        and -inf for padding.

    Returns:
      [B, H, Nq, Dv] in v's dtype, laid out as `output_strides` says. Rows
      whose keys are all masked are NaN.

    Raises:
      ValueError: bad ranks, shapes or dtypes, or a key_bias that varies
        across queries ('key_bias must be constant across queries').
    """
    return torch.ops.vectra.rbf_attention(q, k, v, scale, key_bias)


KERNELS = {'generic': _lib.FLAG_FORCE_GENERIC,
           'decode': _lib.FLAG_FORCE_DECODE,
           'tc': _lib.FLAG_FORCE_TC,
           'small': _lib.FLAG_FORCE_SMALL,
           'small_tc': _lib.FLAG_FORCE_SMALL_TC}


def rbf_attention_with_kernel(q, k, v, scale, key_bias=None,
                              kernel: str = 'auto') -> torch.Tensor:
    """The same operator with the kernel pinned ('generic', 'decode', 'tc',
    'small', 'small_tc').

    Raises ValueError when the pinned kernel cannot run the problem.
    """
    flags = 0 if kernel == 'auto' else KERNELS[kernel]
    return torch.ops.vectra_b200.rbf_attention_with_flags(
        q, k, v, scale, key_bias, flags)


def _describe(t):
    d = _lib.Tensor()
    if t is None:
        return d
    d.data = t.data_ptr() or 0x10000  # never dereferenced by selection
    d.dtype = {torch.float32: _lib.F32, torch.float16: _lib.F16,
               torch.bfloat16: _lib.BF16, torch.float64: _lib.F64}.get(
                   t.dtype, -1)
    d.ndim = t.dim()
    for i in range(t.dim()):
        d.size[i] = t.shape[i]
        d.stride[i] = t.stride(i)
    return d


def kernel_for(q, k, v, scale, key_bias=None, kernel: str = 'auto') -> str:
    """Name of the kernel the operator launches for these tensors
    ('decode', 'tc', 'small_tc', 'small', 'generic' or 'none'); raises
    ValueError when the arguments are invalid. Launches nothing."""
    import ctypes  # pylint: disable=import-outside-toplevel
    a = _lib.Args()
    a.q, a.k, a.v = _describe(q), _describe(k), _describe(v)
    a.scale, a.key_bias = _describe(scale), _describe(key_bias)
    a.out = 0x10000
    st = output_strides(q, v.shape[-1])
    for i in range(4):
        a.out_stride[i] = st[i]
    a.flags = 0 if kernel == 'auto' else KERNELS[kernel]
    res = _lib.LIB.vectra_rbf_select_kernel(ctypes.byref(a))
    if res < 0:
        raise ValueError(_lib.strerror(res))
    return _lib.kernel_name(res)
