"""tensor — device versions of the reference's public tensor ops that sit on
the decode path (src/tensor.rs).  The compute runs in the sm_100a library;
inputs are host arrays (copied in and out by the library) or device buffers
given as raw pointers (anything with a data_ptr() method, e.g. a framework
tensor already on the GPU)."""
from __future__ import annotations

import numpy as np

from . import _lib as L


def scaled_dot_product_attention(q, k, v, n_heads: int, head_dim: int, n_kv_heads: int | None = None):
    """tensor::scaled_dot_product_attention (src/tensor.rs:451-551) for full
    K/V (cache rows first) with GQA: q [q_len, n_heads*head_dim], k/v
    [kv_len, n_kv_heads*head_dim].  Host arrays in, a host f32 array
    [q_len, n_heads*head_dim] out."""
    n_kv_heads = n_kv_heads or n_heads
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    q_len = q.size // (n_heads * head_dim)
    kv_len = k.size // (n_kv_heads * head_dim)
    if q.size != q_len * n_heads * head_dim or k.size != kv_len * n_kv_heads * head_dim or v.size != k.size:
        raise ValueError("q / k / v sizes do not match the head geometry")
    out = np.zeros((q_len, n_heads * head_dim), dtype=np.float32)
    L.check(L.lib().fa_sdpa_host(L.f32_ptr(q), L.f32_ptr(k), L.f32_ptr(v), q_len, kv_len, n_heads, n_kv_heads,
                                 head_dim, L.f32_ptr(out)))
    return out


def scaled_dot_product_attention_device(q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, q_len: int, kv_len: int,
                                        n_heads: int, head_dim: int, n_kv_heads: int | None = None, stream: int = 0):
    """The same on device buffers given as raw device pointers (ints) or
    objects with data_ptr(); enqueued on `stream` (a cudaStream_t as int)."""
    ptr = [p.data_ptr() if hasattr(p, "data_ptr") else int(p) for p in (q_ptr, k_ptr, v_ptr, out_ptr)]
    L.check(L.lib().fa_sdpa(ptr[0], ptr[1], ptr[2], q_len, kv_len, n_heads, n_kv_heads or n_heads, head_dim, ptr[3],
                            stream))
