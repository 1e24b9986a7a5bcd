"""CPU oracle for RBF attention: a NumPy restatement of the reference formulas.

TEST INFRASTRUCTURE ONLY. This module is the checker that the CUDA path is
compared against. Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s
CPU-baseline / reference arm may import it; the product package
`vectra_b200` never does, and no CUDA tensor is ever routed through it.

Every function restates one formulation of Vectra's RBF attention,

    out[b,h,i,:] = sum_j softmax_j(-scale[b,h] * ||q[b,h,i] - k[b,h,j]||^2
                                   + key_bias[b,h,j]) * v[b,h,j,:]

with q [B,H,Nq,D], k [B,H,Nk,D], v [B,H,Nk,Dv], `scale` broadcastable to
[B,H,1,1] and `key_bias` broadcastable to [B,1|H,1,Nk] (0 or -inf for padded
keys). Arrays are NumPy; half-precision inputs are passed as float32 arrays
holding exactly representable values (see `round_to`).

Parity is pinned: tests/golden/make_golden.py ran the reference's own
functions (kernels/vectra_kernels/reference.py) on seeded inputs and stored
their outputs; tests/test_oracle_golden.py checks every function here against
those vectors.
"""

from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634


# ---------------------------------------------------------------------------
# Element rounding (host-side stand-ins for bf16 / fp16 storage).
# ---------------------------------------------------------------------------

def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Rounds float32 values to the nearest bfloat16 (ties to even).

    bfloat16 is the upper 16 bits of an IEEE float32, so rounding adds half
    an ulp of the dropped 16 bits (plus the kept lsb for ties) and truncates.
    NaN stays NaN.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(x)
    out[nan] = np.nan
    return out


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """uint16 bit patterns of float32 values that are already bf16-exact."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    """float32 values of uint16 bf16 bit patterns."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Rounds float values to `dtype` ('f32', 'f16' or 'bf16'), as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == 'f32':
        return x.copy()
    if dtype == 'f16':
        return x.astype(np.float16).astype(np.float32)
    if dtype == 'bf16':
        return round_to_bf16(x)
    raise ValueError(f'unknown dtype {dtype!r}')


# ---------------------------------------------------------------------------
# Broadcasting of the coefficient and the key bias.
# ---------------------------------------------------------------------------

def broadcast_scale(scale, q: np.ndarray, dtype=np.float64) -> np.ndarray:
    """Scale as [B, H, 1, 1].

    Follows kernels/vectra_kernels/reference.py:41-43 (`_broadcast_scale`):
    the coefficient is cast to the compute type and expanded over the
    leading two axes of q.
    """
    s = np.asarray(scale, dtype=dtype)
    while s.ndim < 4:
        s = s[None]
    return np.broadcast_to(s, (*q.shape[:2], 1, 1))


def broadcast_bias(key_bias, q: np.ndarray, n_k: int, dtype=np.float64):
    """Key bias as [B, H, 1, Nk], or None.

    Follows kernels/vectra_kernels/spatial_rbf_attention.py:220-234: the
    bias is left-padded to rank 4, must be constant across queries
    (shape[-2] == 1, else ValueError), and broadcasts over batch and heads.
    """
    if key_bias is None:
        return None
    b = np.asarray(key_bias, dtype=dtype)
    while b.ndim < 4:
        b = b[None]
    if b.shape[-2] != 1:
        raise ValueError('key_bias must be constant across queries')
    return np.broadcast_to(b, (*q.shape[:2], 1, n_k))


def _softmax_last(logits: np.ndarray) -> np.ndarray:
    """Softmax over the last axis; rows that are entirely -inf give NaN.

    This is torch.softmax's behaviour on a fully masked row (max = -inf,
    exp(-inf - -inf) = NaN), which the reference asserts at
    kernels/tests/test_edges.py:74-81.
    """
    with np.errstate(invalid='ignore', over='ignore', divide='ignore'):
        m = logits.max(axis=-1, keepdims=True)
        e = np.exp(logits - m)
        return e / e.sum(axis=-1, keepdims=True)


# ---------------------------------------------------------------------------
# The four reference formulations.
# ---------------------------------------------------------------------------

def expanded_rbf_attention(q, k, v, scale, key_bias=None) -> np.ndarray:
    """Float64 oracle via the Euclidean expansion, clamped at zero.

    Follows kernels/vectra_kernels/reference.py:61-76
    (`expanded_rbf_attention`): ||q||^2 + ||k||^2 - 2 q.k clamped to >= 0,
    times -scale, plus the bias, softmax, times V; everything in float64.
    """
    q64, k64, v64 = (np.asarray(t, dtype=np.float64) for t in (q, k, v))
    q_norm = (q64 * q64).sum(-1, keepdims=True)
    k_norm = (k64 * k64).sum(-1)[..., None, :]
    sq = np.maximum(q_norm + k_norm - 2.0 * (q64 @ np.swapaxes(k64, -1, -2)),
                    0.0)
    logits = -sq * broadcast_scale(scale, q64)
    bias = broadcast_bias(key_bias, q64, k64.shape[-2])
    if bias is not None:
        logits = logits + bias
    return _softmax_last(logits) @ v64


def eager_rbf_attention(q, k, v, scale, key_bias=None,
                        dtype=np.float32) -> np.ndarray:
    """The eager operator chain: broadcast difference, square, sum.

    Follows kernels/vectra_kernels/reference.py:46-58
    (`eager_rbf_attention`): it materialises the [B,H,Nq,Nk,D] difference
    tensor, so it is only used at sizes where that fits comfortably. It is
    computed in `dtype` (float32 by default: the fp32 reference that bf16
    results are compared against).
    """
    qd, kd, vd = (np.asarray(t, dtype=dtype) for t in (q, k, v))
    diff = qd[..., :, None, :] - kd[..., None, :, :]
    sq = (diff * diff).sum(-1)
    logits = -sq * broadcast_scale(scale, qd, dtype)
    bias = broadcast_bias(key_bias, qd, kd.shape[-2], dtype)
    if bias is not None:
        logits = logits + bias
    return (_softmax_last(logits) @ vd).astype(dtype)


def matmul_rbf_attention(q, k, v, scale, key_bias=None) -> np.ndarray:
    """The operator's CPU arithmetic: float32 expansion, clamp, softmax, PV.

    Follows kernels/vectra_kernels/reference.py:79-99
    (`matmul_rbf_attention`). Returns float32; the reference then casts to
    v's dtype, which callers apply with `round_to`.
    """
    qf, kf, vf = (np.asarray(t, dtype=np.float32) for t in (q, k, v))
    q_norm = (qf * qf).sum(-1, keepdims=True)
    k_norm = (kf * kf).sum(-1)[..., None, :]
    sq = np.maximum(q_norm + k_norm - np.float32(2.0) *
                    (qf @ np.swapaxes(kf, -1, -2)), np.float32(0.0))
    logits = -broadcast_scale(scale, qf, np.float32) * sq
    bias = broadcast_bias(key_bias, qf, kf.shape[-2], np.float32)
    if bias is not None:
        logits = logits + bias
    return (_softmax_last(logits) @ vf).astype(np.float32)


def tiled_rbf_attention(q, k, v, scale, key_bias=None, block_q=64,
                        block_k=64) -> np.ndarray:
    """Tile-by-tile online softmax, the streaming kernels' algorithm.

    Follows kernels/vectra_kernels/reference.py:102-161
    (`tiled_rbf_attention`): per query tile a running maximum and running
    sum rescale the accumulator as key tiles stream past; a row whose keys
    so far are all masked keeps a -inf maximum and uses 0 in its place
    (the `safe_max` rule), so exp never sees inf - inf. float32 throughout.
    """
    qf, kf, vf = (np.asarray(t, dtype=np.float32) for t in (q, k, v))
    scale4 = broadcast_scale(scale, qf, np.float32)
    n_q, n_k = qf.shape[-2], kf.shape[-2]
    bias = broadcast_bias(key_bias, qf, n_k, np.float32)
    out = np.empty((*qf.shape[:-1], vf.shape[-1]), dtype=np.float32)
    with np.errstate(invalid='ignore', over='ignore', divide='ignore'):
        for q0 in range(0, n_q, block_q):
            qt = qf[..., q0:q0 + block_q, :]
            q_norm = (qt * qt).sum(-1, keepdims=True)
            rows = qt.shape[-2]
            run_max = np.full((*qf.shape[:2], rows, 1), -np.inf, np.float32)
            run_sum = np.zeros_like(run_max)
            acc = np.zeros((*qf.shape[:2], rows, vf.shape[-1]), np.float32)
            for k0 in range(0, n_k, block_k):
                kt = kf[..., k0:k0 + block_k, :]
                vt = vf[..., k0:k0 + block_k, :]
                k_norm = (kt * kt).sum(-1)[..., None, :]
                dot = qt @ np.swapaxes(kt, -1, -2)
                sq = np.maximum(q_norm + k_norm - np.float32(2.0) * dot,
                                np.float32(0.0))
                logits = -scale4 * sq
                if bias is not None:
                    logits = logits + bias[..., k0:k0 + block_k]
                new_max = np.maximum(run_max,
                                     logits.max(-1, keepdims=True))
                safe = np.where(np.isneginf(new_max), np.float32(0.0),
                                new_max)
                alpha = np.exp(run_max - safe)
                w = np.exp(logits - safe)
                run_sum = run_sum * alpha + w.sum(-1, keepdims=True)
                acc = acc * alpha + w @ vt
                run_max = new_max
            out[..., q0:q0 + rows, :] = acc / run_sum
    return out


# ---------------------------------------------------------------------------
# Helpers shared by the tests and the CPU baseline.
# ---------------------------------------------------------------------------

def reference_output(q, k, v, scale, key_bias=None, out_dtype='f32'):
    """The fp32 reference the CUDA path is compared against.

    The eager formulation (reference.py:46-58) in float32 on the (already
    rounded) inputs, rounded to the output dtype the operator returns
    (v's dtype). Fully masked rows are NaN, as in the reference.
    """
    return round_to(eager_rbf_attention(q, k, v, scale, key_bias), out_dtype)


def sample_planes(q, k, v, scale, key_bias, idx):
    """Restricts an attention problem to batch rows `idx` (for sampling).

    Broadcast dimensions of the scale and the bias (size 1) are kept.
    """
    def pick(t):
        if t is None:
            return None
        t = np.asarray(t)
        while t.ndim < 4:
            t = t[None]
        return t if t.shape[0] == 1 else t[idx]
    return q[idx], k[idx], v[idx], pick(scale), pick(key_bias)
