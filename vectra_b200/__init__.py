"""vectra_b200: Vectra's RBF-attention operator on B200 (sm_100a).

Importing the package registers torch.ops.vectra.rbf_attention with its
CUDA implementation (hand-written kernels in libvectra_rbf.so behind the C
ABI of include/vectra_rbf.h). It raises ImportError if the libraries have
not been built (`python vectra_b200/build.py`).
"""

from vectra_b200 import _lib
from vectra_b200.custom_ops import OP_NAME
from vectra_b200.custom_ops import cuda_available
from vectra_b200.custom_ops import kernel_for
from vectra_b200.custom_ops import rbf_attention
from vectra_b200.custom_ops import rbf_attention_with_kernel

__all__ = ['OP_NAME', 'cuda_available', 'kernel_for', 'rbf_attention',
           'rbf_attention_with_kernel', 'launch_count', 'build_info']

launch_count = _lib.launch_count
build_info = _lib.build_info
