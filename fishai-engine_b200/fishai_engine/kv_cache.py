"""KVCache — src/kv_cache.rs:13-110, device resident and paged (16 positions
per page).  Unlike the reference's Vec<f32>, capacity is fixed at creation
(max_ctx); appends happen inside ModelWeights.forward on the device."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L


class KVCache:
    def __init__(self, model, max_ctx: int = None, n_seq: int = 1, dtype: int = L.KV_F32):
        self.model = model
        cfg = model.config
        self.max_ctx = int(max_ctx or cfg.context_len)
        self.n_seq = n_seq
        self.dtype = dtype
        self._n_layers = cfg.n_layers
        # a tensor-parallel rank caches only the KV heads it holds
        self.kv_dim = getattr(model, "local_kv_heads", cfg.n_kv_heads) * cfg.head_dim
        h = C.c_void_p()
        L.check(L.lib().fa_kv_create(model._h, n_seq, self.max_ctx, dtype, C.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            L.lib().fa_kv_free(h)
            self._h = None

    def n_layers(self) -> int:
        return self._n_layers

    def get(self, layer: int, seq: int = 0):
        """KVCache::get (src/kv_cache.rs:66-69): (k, v) as flat f32 [len * n_kv * head_dim];
        raises IndexError for a bad layer where the reference panics."""
        if layer >= self._n_layers or layer < 0:
            raise IndexError(f"KV cache layer index out of range: {layer} >= {self._n_layers}")
        n = self.seq_len_with_dim(layer, self.kv_dim, seq) * self.kv_dim
        k = np.zeros(max(n, 1), dtype=np.float32)
        v = np.zeros(max(n, 1), dtype=np.float32)
        L.check(L.lib().fa_kv_get(self._h, seq, layer, L.f32_ptr(k), L.f32_ptr(v)))
        return k[:n], v[:n]

    def seq_len(self, layer: int) -> int:
        """KVCache::seq_len (src/kv_cache.rs:75-83) returns 0 in the reference
        whatever the content; kept as is.  Use seq_len_with_dim."""
        if layer >= self._n_layers:
            raise IndexError(f"KV cache layer index out of range: {layer} >= {self._n_layers}")
        return 0

    def seq_len_with_dim(self, layer: int, kv_dim: int, seq: int = 0) -> int:
        """src/kv_cache.rs:90-96"""
        if layer >= self._n_layers:
            raise IndexError(f"KV cache layer index out of range: {layer} >= {self._n_layers}")
        if kv_dim == 0:
            return 0
        n = C.c_uint32()
        L.check(L.lib().fa_kv_seq_len(self._h, seq, C.byref(n)))
        return n.value * self.kv_dim // kv_dim

    def clear(self, seq: int = -1):
        """src/kv_cache.rs:98-103"""
        L.check(L.lib().fa_kv_clear(self._h, seq))
