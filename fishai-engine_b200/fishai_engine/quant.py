"""quant — ggml type ids and dequantisation (src/quant.rs:17-382), on the device."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L

GGML_TYPE_F32, GGML_TYPE_F16, GGML_TYPE_Q4_0, GGML_TYPE_Q4_1 = 0, 1, 2, 3
GGML_TYPE_Q5_0, GGML_TYPE_Q5_1, GGML_TYPE_Q8_0, GGML_TYPE_Q8_1 = 6, 7, 8, 9
GGML_TYPE_Q2_K, GGML_TYPE_Q3_K, GGML_TYPE_Q4_K, GGML_TYPE_Q5_K, GGML_TYPE_Q6_K = 10, 11, 12, 13, 14

_BLOCK = {0: 1, 1: 1, 2: 32, 3: 32, 6: 32, 7: 32, 8: 32, 9: 32, 10: 256, 11: 256, 12: 256, 13: 256, 14: 256}
_SIZE = {0: 4, 1: 2, 2: 18, 3: 20, 6: 22, 7: 24, 8: 34, 9: 40, 10: 84, 11: 110, 12: 144, 13: 176, 14: 210}


def from_u32(v: int):
    """src/quant.rs:34-50"""
    return v if v in _BLOCK else None


def block_size(t: int) -> int:
    """src/quant.rs:345-361"""
    return _BLOCK.get(t, 1)


def type_size(t: int) -> int:
    """src/quant.rs:364-382"""
    return _SIZE.get(t, 4)


def dequantize(data, ggml_type: int, count: int) -> np.ndarray:
    """quant::dequantize (src/quant.rs:312-338), executed by the sm_100a
    dequantisation kernel.  Q4_K and Q6_K are supported in addition to the
    reference's types; short data yields fewer values, as in the reference."""
    buf = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else np.ascontiguousarray(data, dtype=np.uint8)
    out = np.zeros(max(count, 1), dtype=np.float32)
    n = C.c_size_t()
    L.check(L.lib().fa_dequantize(ggml_type, buf.ctypes.data_as(C.c_void_p), buf.size, count, L.f32_ptr(out), C.byref(n)))
    return out[: n.value]
