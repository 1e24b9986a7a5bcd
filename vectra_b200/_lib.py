"""ctypes view of libvectra_rbf.so, the C ABI in include/vectra_rbf.h.

The library is loaded once per process. Importing this module raises
ImportError when the library has not been built: there is no fallback.
"""

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, 'libvectra_rbf.so')
TORCH_EXT_PATH = os.path.join(PKG, '_vectra_rbf_torch.so')

# vectra_dtype
F32, F16, BF16, F64 = 0, 1, 2, 3
# status codes
OK = 0
ERR_NULL, ERR_RANK, ERR_SHAPE, ERR_DTYPE = -1, -2, -3, -4
ERR_SCALE_SHAPE, ERR_BIAS_SHAPE, ERR_BIAS_QUERY = -5, -6, -7
ERR_UNSUPPORTED, ERR_CUDA, ERR_DEVICE, ERR_FORCED = -8, -9, -10, -11
# kernel selection flags
FLAG_FORCE_GENERIC, FLAG_FORCE_DECODE, FLAG_FORCE_TC = 0x1, 0x2, 0x4
FLAG_FORCE_SMALL = 0x10
FLAG_FORCE_SMALL_TC = 0x20
# kernels
KERNEL_NONE, KERNEL_GENERIC, KERNEL_DECODE, KERNEL_TC = 0, 1, 2, 3
KERNEL_SMALL = 5
KERNEL_SMALL_TC = 6

# Every symbol include/vectra_rbf.h declares.
EXPORTED = (
    'vectra_rbf_attention_forward',
    'vectra_rbf_select_kernel',
    'vectra_rbf_kernel_name',
    'vectra_rbf_strerror',
    'vectra_rbf_check_device_errors',
    'vectra_rbf_selftest_wait_timeout',
    'vectra_rbf_launch_count',
    'vectra_rbf_build_info',
)


class Tensor(ctypes.Structure):
    """vectra_tensor."""
    _fields_ = [('data', ctypes.c_void_p), ('dtype', ctypes.c_int32),
                ('ndim', ctypes.c_int32), ('size', ctypes.c_int64 * 4),
                ('stride', ctypes.c_int64 * 4)]


class Args(ctypes.Structure):
    """vectra_rbf_args."""
    _fields_ = [('q', Tensor), ('k', Tensor), ('v', Tensor),
                ('scale', Tensor), ('key_bias', Tensor),
                ('out', ctypes.c_void_p), ('out_stride', ctypes.c_int64 * 4),
                ('flags', ctypes.c_uint32)]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f'{LIB_PATH} is missing: build it with `python '
            'vectra_b200/build.py` (nvcc, sm_100a). CUDA tensors have no CPU '
            'or Triton fallback.')
    lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
    lib.vectra_rbf_attention_forward.argtypes = [ctypes.POINTER(Args),
                                                 ctypes.c_void_p]
    lib.vectra_rbf_attention_forward.restype = ctypes.c_int
    lib.vectra_rbf_select_kernel.argtypes = [ctypes.POINTER(Args)]
    lib.vectra_rbf_select_kernel.restype = ctypes.c_int
    lib.vectra_rbf_kernel_name.argtypes = [ctypes.c_int]
    lib.vectra_rbf_kernel_name.restype = ctypes.c_char_p
    lib.vectra_rbf_strerror.argtypes = [ctypes.c_int]
    lib.vectra_rbf_strerror.restype = ctypes.c_char_p
    lib.vectra_rbf_check_device_errors.argtypes = [ctypes.c_void_p]
    lib.vectra_rbf_check_device_errors.restype = ctypes.c_int
    lib.vectra_rbf_selftest_wait_timeout.argtypes = [ctypes.c_void_p]
    lib.vectra_rbf_selftest_wait_timeout.restype = ctypes.c_int
    lib.vectra_rbf_launch_count.argtypes = []
    lib.vectra_rbf_launch_count.restype = ctypes.c_uint64
    lib.vectra_rbf_build_info.argtypes = []
    lib.vectra_rbf_build_info.restype = ctypes.c_char_p
    return lib


LIB = _load()


def strerror(status: int) -> str:
    return LIB.vectra_rbf_strerror(status).decode()


def kernel_name(kernel: int) -> str:
    return LIB.vectra_rbf_kernel_name(kernel).decode()


def launch_count() -> int:
    """Kernels this process launched through the library."""
    return int(LIB.vectra_rbf_launch_count())


def build_info() -> str:
    return LIB.vectra_rbf_build_info().decode()


def check_device_errors(stream_handle: int = 0) -> int:
    """Synchronises the stream and reads/clears the device error word."""
    return int(LIB.vectra_rbf_check_device_errors(
        ctypes.c_void_p(stream_handle)))


def selftest_wait_timeout(stream_handle: int = 0) -> int:
    """Launches the failure-path self-test kernel (a bounded wait that runs
    out after about 2 s); see vectra_rbf_selftest_wait_timeout."""
    return int(LIB.vectra_rbf_selftest_wait_timeout(
        ctypes.c_void_p(stream_handle)))
