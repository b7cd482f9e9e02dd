"""BpeTokenizer — src/tokenizer.rs:148-600, in the C++ library (host code,
no device): GGUF vocabulary, BPE merges by rank, <0xNN> byte fallback,
special tokens.  TokenType values follow src/tokenizer.rs:27-40."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

from . import _lib as L

NORMAL, UNKNOWN, BYTE, CONTROL, USER_DEFINED = 0, 1, 2, 3, 4


class fa_tokenizer_config(C.Structure):
    _fields_ = [("bos_token_id", C.c_int64), ("eos_token_id", C.c_int64), ("eot_token_id", C.c_int64),
                ("eom_token_id", C.c_int64), ("unk_token_id", C.c_int64), ("add_bos", C.c_int32),
                ("add_eos", C.c_int32), ("add_space_prefix", C.c_int32),
                ("remove_special_whitespaces", C.c_int32), ("prepend_bos", C.c_int32)]


@dataclass
class TokenizerConfig:
    """src/tokenizer.rs:107-144 (None for an absent id)"""
    bos_token_id: Optional[int] = None
    eos_token_id: Optional[int] = None
    eot_token_id: Optional[int] = None
    eom_token_id: Optional[int] = None
    unk_token_id: Optional[int] = None
    add_bos: bool = False
    add_eos: bool = False
    add_space_prefix: bool = False
    remove_special_whitespaces: bool = False
    prepend_bos: bool = False

    def _c(self):
        n = lambda v: -1 if v is None else int(v)  # noqa: E731
        return fa_tokenizer_config(n(self.bos_token_id), n(self.eos_token_id), n(self.eot_token_id),
                                   n(self.eom_token_id), n(self.unk_token_id), int(self.add_bos), int(self.add_eos),
                                   int(self.add_space_prefix), int(self.remove_special_whitespaces),
                                   int(self.prepend_bos))

    @staticmethod
    def _from_c(c):
        o = lambda v: None if v < 0 else int(v)  # noqa: E731
        return TokenizerConfig(o(c.bos_token_id), o(c.eos_token_id), o(c.eot_token_id), o(c.eom_token_id),
                               o(c.unk_token_id), bool(c.add_bos), bool(c.add_eos), bool(c.add_space_prefix),
                               bool(c.remove_special_whitespaces), bool(c.prepend_bos))


class BpeTokenizer:
    def __init__(self, handle):
        self._h = handle

    @classmethod
    def from_gguf(cls, tokens: Sequence[str], scores: Sequence[float] = (), token_types: Sequence[int] = (),
                  merges: Optional[str] = None, config: Optional[TokenizerConfig] = None) -> "BpeTokenizer":
        """BpeTokenizer::from_gguf (src/tokenizer.rs:202-286) from the GGUF's arrays"""
        enc = [t.encode("utf-8") for t in tokens]
        arr = (C.c_char_p * max(len(enc), 1))(*enc)
        sc = np.ascontiguousarray(np.asarray(scores, dtype=np.float32))
        ty = np.ascontiguousarray(np.asarray(token_types, dtype=np.int32))
        cfg = (config or TokenizerConfig())._c()
        h = C.c_void_p()
        L.check(L.lib().fa_tokenizer_create(arr, len(enc), sc.ctypes.data_as(C.POINTER(C.c_float)), sc.size,
                                            ty.ctypes.data_as(C.POINTER(C.c_int32)), ty.size,
                                            merges.encode("utf-8") if merges is not None else None, C.byref(cfg),
                                            C.byref(h)))
        return cls(h)

    @classmethod
    def from_gguf_file(cls, gguf) -> "BpeTokenizer":
        """the tokenizer a GGUF file carries (tokenizer.ggml.* keys)"""
        from .gguf import GGUFFile

        g = gguf if isinstance(gguf, GGUFFile) else GGUFFile.open(str(gguf))
        h = C.c_void_p()
        L.check(L.lib().fa_tokenizer_from_gguf(g._h, C.byref(h)))
        return cls(h)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            L.lib().fa_tokenizer_free(h)
            self._h = None

    def _encode(self, text: str, add_special: bool, with_special: bool) -> List[int]:
        b = text.encode("utf-8")
        n = C.c_size_t()
        L.check(L.lib().fa_tokenizer_encode(self._h, b, len(b), int(add_special), int(with_special), None, 0,
                                            C.byref(n)))
        ids = np.zeros(max(n.value, 1), dtype=np.uint32)
        L.check(L.lib().fa_tokenizer_encode(self._h, b, len(b), int(add_special), int(with_special),
                                            ids.ctypes.data_as(C.POINTER(C.c_uint32)), ids.size, C.byref(n)))
        return ids[: n.value].tolist()

    def encode(self, text: str, add_special: bool) -> List[int]:
        """src/tokenizer.rs:290-344"""
        return self._encode(text, add_special, False)

    def encode_with_special(self, text: str) -> List[int]:
        """src/tokenizer.rs:347-391"""
        return self._encode(text, False, True)

    def decode(self, ids: Sequence[int]) -> str:
        """src/tokenizer.rs:394-408"""
        a, p = L.u32_array(list(ids) or [0])
        n = len(ids)
        ln = C.c_size_t()
        L.check(L.lib().fa_tokenizer_decode(self._h, p, n, None, 0, C.byref(ln)))
        buf = C.create_string_buffer(ln.value + 1)
        L.check(L.lib().fa_tokenizer_decode(self._h, p, n, buf, ln.value + 1, C.byref(ln)))
        return buf.raw[: ln.value].decode("utf-8", errors="replace")

    def token_to_piece(self, token_id: int) -> Optional[str]:
        """src/tokenizer.rs:411-418 (None outside the vocabulary)"""
        if token_id < 0 or token_id >= self.vocab_size():
            return None
        ln, ty = C.c_size_t(), C.c_int32()
        L.check(L.lib().fa_tokenizer_piece(self._h, token_id, None, 0, C.byref(ln), C.byref(ty)))
        buf = C.create_string_buffer(ln.value + 1)
        L.check(L.lib().fa_tokenizer_piece(self._h, token_id, buf, ln.value + 1, C.byref(ln), C.byref(ty)))
        return buf.raw[: ln.value].decode("utf-8", errors="replace")

    def token_type(self, token_id: int) -> int:
        ln, ty = C.c_size_t(), C.c_int32()
        L.check(L.lib().fa_tokenizer_piece(self._h, token_id, None, 0, C.byref(ln), C.byref(ty)))
        return ty.value

    def byte_token(self, b: int) -> int:
        out = C.c_uint32()
        L.check(L.lib().fa_tokenizer_byte_token(self._h, b, C.byref(out)))
        return out.value

    def _info(self):
        v = C.c_uint32()
        c = fa_tokenizer_config()
        L.check(L.lib().fa_tokenizer_info(self._h, C.byref(v), C.byref(c)))
        return v.value, TokenizerConfig._from_c(c)

    def vocab_size(self) -> int:
        return self._info()[0]

    @property
    def config(self) -> TokenizerConfig:
        return self._info()[1]

    def bos_token(self) -> Optional[int]:
        return self.config.bos_token_id

    def eos_token(self) -> Optional[int]:
        return self.config.eos_token_id
