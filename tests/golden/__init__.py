"""Golden vectors produced by the reference's own functions.

`load(name)` returns one case as a dict of float32/float64 NumPy arrays
(half-precision inputs widened by value, which is exact) plus its dtype.
"""

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def names():
    with open(os.path.join(HERE, 'index.json'), encoding='utf-8') as f:
        return sorted(json.load(f))


def _widen(a: np.ndarray) -> np.ndarray:
    if a.dtype == np.uint16:  # bfloat16 bit patterns
        return (a.astype(np.uint32) << 16).view(np.float32)
    if a.dtype == np.float16:
        return a.astype(np.float32)
    return a


def load(name: str) -> dict:
    with np.load(os.path.join(HERE, f'{name}.npz')) as z:
        case = {key: z[key] for key in z.files}
    meta = json.loads(bytes(case.pop('meta')).decode())
    out = {key: (val if key == 'expanded' else _widen(val))
           for key, val in case.items()}
    out['dtype'] = meta['dtype']
    out.setdefault('bias', None)
    return out
