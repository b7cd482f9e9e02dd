"""GGUFFile — src/gguf.rs:438-758 over the C ABI (host-side parser)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L
from .quant import dequantize


class TensorInfo:
    """src/gguf.rs:219-244"""

    def __init__(self, name, n_dims, dims, ggml_type, offset):
        self.name, self.n_dims, self.dims, self.ggml_type, self.offset = name, n_dims, list(dims), ggml_type, offset

    def nelement(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    def shape(self):
        return list(self.dims)


class GGUFFile:
    def __init__(self, handle, path):
        self._h = handle
        self.path = path

    @classmethod
    def open(cls, path: str) -> "GGUFFile":
        """GGUFFile::open (src/gguf.rs:438-561); raises FishaiError where the reference returns Err."""
        h = C.c_void_p()
        L.check(L.lib().fa_gguf_open(str(path).encode(), C.byref(h)))
        return cls(h, str(path))

    def close(self):
        if self._h:
            L.lib().fa_gguf_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def version(self) -> int:
        v = C.c_uint32()
        L.check(L.lib().fa_gguf_version(self._h, C.byref(v)))
        return v.value

    @property
    def alignment(self) -> int:
        v = C.c_uint64()
        L.check(L.lib().fa_gguf_alignment(self._h, C.byref(v)))
        return v.value

    def tensor_count(self) -> int:
        n = C.c_size_t()
        L.check(L.lib().fa_gguf_tensor_count(self._h, C.byref(n)))
        return n.value

    def tensor_names(self):
        out = []
        for i in range(self.tensor_count()):
            buf = C.create_string_buffer(4096)
            L.check(L.lib().fa_gguf_tensor_at(self._h, i, buf, 4096, None, None, None, None))
            out.append(buf.value.decode())
        return out

    def tensor_info(self, name: str):
        nd, t, off = C.c_uint32(), C.c_uint32(), C.c_uint64()
        dims = (C.c_uint64 * 4)()
        rc = L.lib().fa_gguf_tensor_info(self._h, name.encode(), C.byref(nd), dims, C.byref(t), C.byref(off))
        if rc != L.OK:
            return None
        return TensorInfo(name, nd.value, [dims[i] for i in range(nd.value)], t.value, off.value)

    def read_tensor_data(self, info) -> bytes:
        name = info.name if isinstance(info, TensorInfo) else info
        size = C.c_size_t()
        L.check(L.lib().fa_gguf_read_tensor_data(self._h, name.encode(), None, 0, C.byref(size)))
        if size.value == 0:
            return b""
        buf = (C.c_uint8 * size.value)()
        L.check(L.lib().fa_gguf_read_tensor_data(self._h, name.encode(), buf, size.value, C.byref(size)))
        return bytes(buf)

    def read_tensor_data_f32(self, info) -> np.ndarray:
        """read_tensor_data + quant::dequantize (src/gguf.rs:683-689), dequantised on the device."""
        info = info if isinstance(info, TensorInfo) else self.tensor_info(info)
        raw = self.read_tensor_data(info)
        if not raw:
            raise L.FishaiError(L.ERR_GGUF, f"tensor '{info.name}' has no data")
        return dequantize(raw, info.ggml_type, info.nelement())

    def _meta(self, fn, ctype, key):
        v, found = ctype(), C.c_int()
        L.check(fn(self._h, key.encode(), C.byref(v), C.byref(found)))
        return v.value if found.value else None

    def metadata_u64(self, key):
        return self._meta(L.lib().fa_gguf_meta_u64, C.c_uint64, key)

    def metadata_i64(self, key):
        return self._meta(L.lib().fa_gguf_meta_i64, C.c_int64, key)

    def metadata_f32(self, key):
        return self._meta(L.lib().fa_gguf_meta_f32, C.c_float, key)

    def metadata_bool(self, key):
        v = self._meta(L.lib().fa_gguf_meta_bool, C.c_int, key)
        return None if v is None else bool(v)

    def metadata_string(self, key):
        buf, found = C.create_string_buffer(1 << 16), C.c_int()
        L.check(L.lib().fa_gguf_meta_string(self._h, key.encode(), buf, 1 << 16, C.byref(found)))
        return buf.value.decode(errors="replace") if found.value else None

    def vocab_size(self):
        """src/gguf.rs:748-758"""
        v, found = C.c_uint64(), C.c_int()
        L.check(L.lib().fa_gguf_vocab_size(self._h, C.byref(v), C.byref(found)))
        return v.value if found.value else None

    # architecture accessors, src/gguf.rs:698-746
    def model_architecture(self):
        return self.metadata_string("general.architecture")

    def _arch_u64(self, suffix):
        a = self.model_architecture()
        return None if a is None else self.metadata_u64(f"{a}.{suffix}")

    def context_length(self):
        return self._arch_u64("context_length")

    def embedding_length(self):
        return self._arch_u64("embedding_length")

    def head_count(self):
        return self._arch_u64("attention.head_count")

    def head_count_kv(self):
        return self._arch_u64("attention.head_count_kv")

    def layer_count(self):
        return self._arch_u64("block_count")
