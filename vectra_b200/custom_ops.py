"""torch.ops.vectra.rbf_attention on B200: the reference operator, re-backed.

Mirrors the reference module kernels/vectra_kernels/custom_ops.py: the same
operator name (`OP_NAME`, :44), the same schema (:52-59), the same fake
implementation (:88-97), and a CUDA implementation (:75-85) that is now the
C++ binding in _vectra_rbf_torch.so calling hand-written sm_100a kernels
through libvectra_rbf.so. Differences from the reference, on purpose:

* There is no Triton path and no "CUDA without Triton -> CPU arithmetic"
  fallback (custom_ops.py:39-42,83-84): if the extension is missing,
  importing this module raises.
* There is no CPU implementation: the operator runs on CUDA tensors only and
  raises NotImplementedError for CPU tensors. The reference's CPU
  arithmetic (reference.matmul_rbf_attention) is the oracle here, not
  product code.

Typical usage (unchanged):

    out = torch.ops.vectra.rbf_attention(q, k, v, scale, key_bias)
"""

import torch

from vectra_b200 import _lib

OP_NAME = 'vectra::rbf_attention'

torch.ops.load_library(_lib.TORCH_EXT_PATH)


@torch.library.register_fake(OP_NAME)
def _rbf_attention_fake(q, k, v, scale, key_bias=None):
    del k, scale, key_bias  # Only the output shape matters while tracing.
    return q.new_empty((*q.shape[:-1], v.shape[-1]), dtype=v.dtype)


@torch.library.register_fake('vectra_b200::rbf_attention_with_flags')
def _rbf_attention_with_flags_fake(q, k, v, scale, key_bias, flags):
    del k, scale, key_bias, flags
    return q.new_empty((*q.shape[:-1], v.shape[-1]), dtype=v.dtype)


def cuda_available() -> bool:
    """Whether the B200 kernels can run here (the reference's
    `triton_available`, custom_ops.py:47-49)."""
    return torch.cuda.is_available()


def rbf_attention(q, k, v, scale, key_bias=None) -> torch.Tensor:
    """Fused RBF attention: softmax(-scale * ||q - k||^2 + key_bias) @ v.

    Args:
      q: [B, H, Nq, D] CUDA tensor (float32, float16 or bfloat16), any
        strides.
      k: [B, H, Nk, D], same dtype.
      v: [B, H, Nk, Dv], same dtype.
      scale: Broadcastable to [B, H, 1, 1]; the RBF coefficient
        1 / (2 sigma^2). Zero and negative values are legal.
      key_bias: Optional, broadcastable to [B, 1|H, 1, Nk]; 0 for real keys
        and -inf for padding.

    Returns:
      [B, H, Nq, Dv] in v's dtype. Rows whose keys are all masked are NaN.

    Raises:
      ValueError: bad ranks, shapes or dtypes, or a key_bias that varies
        across queries ('key_bias must be constant across queries').
    """
    return torch.ops.vectra.rbf_attention(q, k, v, scale, key_bias)


KERNELS = {'generic': _lib.FLAG_FORCE_GENERIC,
           'decode': _lib.FLAG_FORCE_DECODE,
           'decode_mma': _lib.FLAG_FORCE_DECODE_MMA,
           'tc': _lib.FLAG_FORCE_TC,
           'small': _lib.FLAG_FORCE_SMALL}


def rbf_attention_with_kernel(q, k, v, scale, key_bias=None,
                              kernel: str = 'auto') -> torch.Tensor:
    """The same operator with the kernel pinned ('generic', 'decode',
    'decode_mma', 'tc', 'small').

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
    ('decode', 'decode_mma', 'tc', 'small', 'generic' or 'none'); raises
    ValueError when the arguments are invalid. Launches nothing."""
    import ctypes  # pylint: disable=import-outside-toplevel
    a = _lib.Args()
    a.q, a.k, a.v = _describe(q), _describe(k), _describe(v)
    a.scale, a.key_bias = _describe(scale), _describe(key_bias)
    a.out = 0x10000
    dv = v.shape[-1]
    st = [q.shape[1] * q.shape[2] * dv, q.shape[2] * dv, dv, 1]
    for i in range(4):
        a.out_stride[i] = st[i]
    a.flags = 0 if kernel == 'auto' else KERNELS[kernel]
    res = _lib.LIB.vectra_rbf_select_kernel(ctypes.byref(a))
    if res < 0:
        raise ValueError(_lib.strerror(res))
    return _lib.kernel_name(res)
