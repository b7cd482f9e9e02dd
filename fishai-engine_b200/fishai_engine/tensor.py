"""tensor — device versions of the reference's public tensor ops that sit on
the decode path (src/tensor.rs).  Buffers are torch CUDA tensors (plumbing
only); the compute runs in the sm_100a library."""
from __future__ import annotations

import math

from . import _lib as L


def _dev_f32(t):
    import torch

    if not isinstance(t, torch.Tensor):
        t = torch.as_tensor(t)
    return t.to(device="cuda", dtype=torch.float32).contiguous()


def scaled_dot_product_attention(q, k, v, n_heads: int, head_dim: int, n_kv_heads: int | None = None):
    """tensor::scaled_dot_product_attention (src/tensor.rs:451-551) for full
    K/V (cache rows first) with GQA: q [q_len, n_heads*head_dim], k/v
    [kv_len, n_kv_heads*head_dim].  Returns a CUDA tensor like q."""
    import torch

    n_kv_heads = n_kv_heads or n_heads
    q, k, v = _dev_f32(q), _dev_f32(k), _dev_f32(v)
    q_len = q.numel() // (n_heads * head_dim)
    kv_len = k.numel() // (n_kv_heads * head_dim)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream().cuda_stream
    L.check(L.lib().fa_sdpa(q.data_ptr(), k.data_ptr(), v.data_ptr(), q_len, kv_len, n_heads, n_kv_heads, head_dim,
                            out.data_ptr(), stream))
    return out
