"""ORACLE — test infrastructure only.

ctypes front end to oracle/build/liboracle.so, the C restatement of the
fishai-engine reference CPU path (see fa_oracle.h for the deviations D1-D4).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only as the test oracle or the timed CPU baseline.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "liboracle.so")
_lib = None

F32 = 0
F16 = 1
Q4_0 = 2
Q4_1 = 3
Q5_0 = 6
Q8_0 = 8
Q4_K = 12
Q6_K = 14


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc only, seconds)."""
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(
        os.path.getmtime(os.path.join(_HERE, f)) for f in ("fa_oracle.c", "fa_oracle.h")
    ):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class _Cfg(C.Structure):
    _fields_ = [
        ("n_layers", C.c_size_t), ("n_heads", C.c_size_t), ("n_kv_heads", C.c_size_t),
        ("head_dim", C.c_size_t), ("n_embd", C.c_size_t), ("vocab_size", C.c_size_t),
        ("context_len", C.c_size_t), ("ffn_dim_multiplier", C.c_float), ("norm_eps", C.c_float),
        ("rope_base", C.c_float), ("rope_freq_dim", C.c_size_t), ("n_ff", C.c_size_t),
        ("n_ff_used", C.c_size_t), ("n_ff_deviation", C.c_int), ("tied_output", C.c_int),
    ]


class _SamplerCfg(C.Structure):
    _fields_ = [
        ("temperature", C.c_float), ("top_k", C.c_size_t), ("top_p", C.c_float),
        ("repetition_penalty", C.c_float), ("frequency_penalty", C.c_float),
        ("presence_penalty", C.c_float),
    ]


class _GenCfg(C.Structure):
    _fields_ = [
        ("max_tokens", C.c_size_t), ("temperature", C.c_float), ("top_k", C.c_size_t),
        ("top_p", C.c_float), ("repetition_penalty", C.c_float),
        ("stop_ids", C.POINTER(C.c_uint32)), ("n_stop", C.c_size_t), ("seed", C.c_uint64),
        ("fast", C.c_int),
    ]


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(build())
        L = _lib
        vp, sz, fp, u8p, u32p = C.c_void_p, C.c_size_t, C.POINTER(C.c_float), C.POINTER(C.c_uint8), C.POINTER(C.c_uint32)
        L.or_f16_to_f32.argtypes = [C.c_uint16]; L.or_f16_to_f32.restype = C.c_float
        L.or_f32_to_f16.argtypes = [C.c_float]; L.or_f32_to_f16.restype = C.c_uint16
        L.or_block_size.argtypes = [C.c_int]; L.or_block_size.restype = sz
        L.or_type_size.argtypes = [C.c_int]; L.or_type_size.restype = sz
        L.or_dequantize.argtypes = [u8p, sz, C.c_int, sz, fp]; L.or_dequantize.restype = C.c_long
        L.or_quantize_q4_0.argtypes = [fp, sz, u8p]; L.or_quantize_q4_0.restype = sz
        L.or_quantize_q8_0.argtypes = [fp, sz, u8p]; L.or_quantize_q8_0.restype = sz
        L.or_matmul.argtypes = [fp, fp, sz, sz, sz, fp]
        L.or_rms_norm.argtypes = [fp, fp, sz, C.c_float, fp]
        L.or_silu.argtypes = [fp, sz, fp]
        L.or_softmax_inplace.argtypes = [fp, sz]
        L.or_rope_emb.argtypes = [sz, sz, C.c_float, fp]
        L.or_apply_rope_to_tensor.argtypes = [fp, sz, sz, sz, sz, C.c_float]
        L.or_sdpa.argtypes = [fp, fp, fp, sz, sz, sz, sz, fp]
        L.or_philox4x32_10.argtypes = [u32p, u32p, u32p]
        L.or_philox_uniform.argtypes = [C.c_uint64, C.c_uint64]; L.or_philox_uniform.restype = C.c_float
        L.or_gguf_open.argtypes = [C.c_char_p, C.c_char_p, sz]; L.or_gguf_open.restype = vp
        L.or_gguf_close.argtypes = [vp]
        L.or_gguf_version.argtypes = [vp]; L.or_gguf_version.restype = C.c_uint32
        L.or_gguf_alignment.argtypes = [vp]; L.or_gguf_alignment.restype = C.c_uint64
        L.or_gguf_tensor_count.argtypes = [vp]; L.or_gguf_tensor_count.restype = sz
        L.or_gguf_tensor_name.argtypes = [vp, sz]; L.or_gguf_tensor_name.restype = C.c_char_p
        L.or_gguf_tensor_info.argtypes = [vp, C.c_char_p, u32p, C.POINTER(C.c_uint64), u32p, C.POINTER(C.c_uint64)]
        L.or_gguf_tensor_info.restype = C.c_int
        L.or_gguf_read_tensor_data.argtypes = [vp, C.c_char_p, u8p, sz]; L.or_gguf_read_tensor_data.restype = sz
        L.or_gguf_meta_u64.argtypes = [vp, C.c_char_p, C.POINTER(C.c_uint64)]; L.or_gguf_meta_u64.restype = C.c_int
        L.or_gguf_meta_i64.argtypes = [vp, C.c_char_p, C.POINTER(C.c_int64)]; L.or_gguf_meta_i64.restype = C.c_int
        L.or_gguf_meta_f32.argtypes = [vp, C.c_char_p, fp]; L.or_gguf_meta_f32.restype = C.c_int
        L.or_gguf_meta_bool.argtypes = [vp, C.c_char_p, C.POINTER(C.c_int)]; L.or_gguf_meta_bool.restype = C.c_int
        L.or_gguf_meta_string.argtypes = [vp, C.c_char_p, C.c_char_p, sz]; L.or_gguf_meta_string.restype = C.c_int
        L.or_gguf_vocab_size.argtypes = [vp, C.POINTER(C.c_uint64)]; L.or_gguf_vocab_size.restype = C.c_int
        L.or_config_from_gguf.argtypes = [vp, C.POINTER(_Cfg), C.c_char_p, sz]; L.or_config_from_gguf.restype = C.c_int
        L.or_config_n_ff.argtypes = [sz, C.c_float]; L.or_config_n_ff.restype = sz
        L.or_model_load.argtypes = [C.c_char_p, C.c_int, C.c_char_p, sz]; L.or_model_load.restype = vp
        L.or_model_free.argtypes = [vp]
        L.or_model_config.argtypes = [vp, C.POINTER(_Cfg)]
        L.or_model_set_threads.argtypes = [vp, C.c_int]
        L.or_kv_new.argtypes = [vp, sz, C.c_int]; L.or_kv_new.restype = vp
        L.or_kv_free.argtypes = [vp]
        L.or_kv_clear.argtypes = [vp]
        L.or_kv_len.argtypes = [vp]; L.or_kv_len.restype = sz
        L.or_kv_get.argtypes = [vp, sz, fp, fp]; L.or_kv_get.restype = C.c_int
        L.or_forward.argtypes = [vp, u32p, sz, sz, vp, fp, fp, C.c_int]; L.or_forward.restype = C.c_int
        L.or_prefill.argtypes = [vp, u32p, sz, sz, vp, fp, fp]; L.or_prefill.restype = C.c_int
        L.or_sampler_new.argtypes = [C.POINTER(_SamplerCfg)]; L.or_sampler_new.restype = vp
        L.or_sampler_free.argtypes = [vp]
        L.or_sampler_sample.argtypes = [vp, fp, sz, C.c_float, C.POINTER(C.c_int)]; L.or_sampler_sample.restype = sz
        L.or_sampler_observe.argtypes = [vp, sz]
        L.or_sampler_reset.argtypes = [vp]
        L.or_sampler_freq.argtypes = [vp, sz]; L.or_sampler_freq.restype = sz
        L.or_softmax_probs.argtypes = [fp, sz, fp]
        L.or_top_k_filter.argtypes = [fp, sz, sz, fp]
        L.or_top_p_filter.argtypes = [fp, sz]
        L.or_categorical_sample.argtypes = [fp, sz, C.c_float]; L.or_categorical_sample.restype = sz
        L.or_argmax.argtypes = [fp, sz]; L.or_argmax.restype = sz
        L.or_generate.argtypes = [vp, C.POINTER(_GenCfg), u32p, sz, u32p, sz, C.c_int]; L.or_generate.restype = C.c_long
        L.or_time_layer.argtypes = [vp, sz, C.POINTER(C.c_double)]; L.or_time_layer.restype = C.c_double
        L.or_time_token.argtypes = [vp, vp, C.c_uint32, sz, sz, C.POINTER(C.c_double)]
        L.or_time_token.restype = C.c_long
        L.or_kv_fill_synthetic.argtypes = [vp, sz, C.c_uint64]
        L.or_kv_set.argtypes = [vp, sz, fp, fp, sz]; L.or_kv_set.restype = C.c_int
    return _lib


class _SynthSpec(C.Structure):  # fa_synth_spec of include/fishai_cuda.h
    _fields_ = [("n_layers", C.c_uint32), ("n_embd", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
                ("n_ff", C.c_uint32), ("vocab", C.c_uint32), ("context_len", C.c_uint32), ("rope_base", C.c_float),
                ("norm_eps", C.c_float), ("sigma", C.c_float), ("type_embd", C.c_int32), ("type_q", C.c_int32),
                ("type_k", C.c_int32), ("type_v", C.c_int32), ("type_o", C.c_int32), ("type_gate", C.c_int32),
                ("type_up", C.c_int32), ("type_down", C.c_int32), ("type_out", C.c_int32), ("threads", C.c_uint32)]


_synth = None


def write_gguf(path: str, seed: int, threads: int = 0, **fields) -> str:
    """The package's synthetic GGUF writer through oracle/build/libsynth.so
    (host code only; byte-identical to fa_synth_write), for callers that must
    not load the CUDA library: the CPU reference arm of bench.py."""
    global _synth
    if _synth is None:
        build()
        _synth = C.CDLL(os.path.join(_HERE, "build", "libsynth.so"))
        _synth.or_synth_write.argtypes = [C.c_char_p, C.POINTER(_SynthSpec), C.c_uint64]
        _synth.or_synth_write.restype = C.c_int
        _synth.or_synth_last_error.argtypes = [C.c_char_p, C.c_size_t]
        _synth.or_synth_last_error.restype = C.c_size_t
    s = _SynthSpec()
    s.threads = threads
    s.type_out = fields.pop("type_out", -1)
    for k, v in fields.items():
        setattr(s, k, v)
    if _synth.or_synth_write(str(path).encode(), C.byref(s), seed):
        buf = C.create_string_buffer(512)
        _synth.or_synth_last_error(buf, 512)
        raise ValueError(buf.value.decode())
    return str(path)


def _f(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(C.POINTER(C.c_float))


def _u8(a):
    a = np.ascontiguousarray(a, dtype=np.uint8)
    return a, a.ctypes.data_as(C.POINTER(C.c_uint8))


def _u32(a):
    a = np.ascontiguousarray(a, dtype=np.uint32)
    return a, a.ctypes.data_as(C.POINTER(C.c_uint32))


# ---------------- quant ----------------
def f16_to_f32(h: int) -> float:
    return lib().or_f16_to_f32(h)


def f32_to_f16(x: float) -> int:
    return lib().or_f32_to_f16(x)


def block_size(t: int) -> int:
    return lib().or_block_size(t)


def type_size(t: int) -> int:
    return lib().or_type_size(t)


def dequantize(data, ggml_type: int, count: int) -> np.ndarray:
    """quant::dequantize; raises ValueError where the reference returns Err."""
    d, dp = _u8(np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else data)
    out = np.zeros(max(count, 1), dtype=np.float32)
    _, op = _f(out)
    n = lib().or_dequantize(dp, d.size, ggml_type, count, out.ctypes.data_as(C.POINTER(C.c_float)))
    if n == -1:
        raise ValueError(f"Unsupported ggml type for dequantization: {ggml_type}")
    if n == -2:
        raise ValueError("Not enough data for F32")
    return out[:n]


def quantize_q4_0(values) -> bytes:
    v, vp = _f(values)
    out = np.zeros(((v.size + 31) // 32) * 18, dtype=np.uint8)
    n = lib().or_quantize_q4_0(vp, v.size, out.ctypes.data_as(C.POINTER(C.c_uint8)))
    return out[:n].tobytes()


def quantize_q8_0(values) -> bytes:
    v, vp = _f(values)
    out = np.zeros(((v.size + 31) // 32) * 34, dtype=np.uint8)
    n = lib().or_quantize_q8_0(vp, v.size, out.ctypes.data_as(C.POINTER(C.c_uint8)))
    return out[:n].tobytes()


# ---------------- tensor ----------------
def matmul(a, b, m, k, n):
    a, ap = _f(a)
    b, bp = _f(b)
    c = np.zeros(m * n, dtype=np.float32)
    lib().or_matmul(ap, bp, m, k, n, c.ctypes.data_as(C.POINTER(C.c_float)))
    return c


def rms_norm(x, w, eps):
    x, xp = _f(x)
    w, wp = _f(w)
    y = np.zeros_like(x)
    lib().or_rms_norm(xp, wp, x.size, eps, y.ctypes.data_as(C.POINTER(C.c_float)))
    return y


def silu(x):
    x, xp = _f(x)
    y = np.zeros_like(x)
    lib().or_silu(xp, x.size, y.ctypes.data_as(C.POINTER(C.c_float)))
    return y


def rope_emb(pos, dim, base):
    e = np.zeros(dim, dtype=np.float32)
    lib().or_rope_emb(pos, dim, base, e.ctypes.data_as(C.POINTER(C.c_float)))
    return e


def apply_rope_to_tensor(data, n_h, head_dim, pos, base):
    d = np.array(data, dtype=np.float32).copy()
    lib().or_apply_rope_to_tensor(d.ctypes.data_as(C.POINTER(C.c_float)), d.size, n_h, head_dim, pos, base)
    return d


def sdpa(q, k, v, n_heads, head_dim):
    q, qp = _f(q)
    k, kp = _f(k)
    v, vp = _f(v)
    qd = n_heads * head_dim
    out = np.zeros(q.size, dtype=np.float32)
    lib().or_sdpa(qp, kp, vp, q.size // qd, k.size // qd, n_heads, head_dim, out.ctypes.data_as(C.POINTER(C.c_float)))
    return out


def philox4x32_10(ctr, key):
    c, cp = _u32(ctr)
    k, kp = _u32(key)
    o = np.zeros(4, dtype=np.uint32)
    lib().or_philox4x32_10(cp, kp, o.ctypes.data_as(C.POINTER(C.c_uint32)))
    return o


def philox_uniform(seed: int, step: int) -> float:
    return lib().or_philox_uniform(seed, step)


# ---------------- gguf ----------------
class GGUF:
    def __init__(self, path: str):
        err = C.create_string_buffer(512)
        self.h = lib().or_gguf_open(path.encode(), err, 512)
        if not self.h:
            raise ValueError(err.value.decode())

    def close(self):
        if self.h:
            lib().or_gguf_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    @property
    def version(self):
        return lib().or_gguf_version(self.h)

    @property
    def alignment(self):
        return lib().or_gguf_alignment(self.h)

    def tensor_names(self):
        L = lib()
        return [L.or_gguf_tensor_name(self.h, i).decode() for i in range(L.or_gguf_tensor_count(self.h))]

    def tensor_info(self, name):
        nd, t = C.c_uint32(), C.c_uint32()
        dims = (C.c_uint64 * 4)()
        off = C.c_uint64()
        if lib().or_gguf_tensor_info(self.h, name.encode(), C.byref(nd), dims, C.byref(t), C.byref(off)):
            return None
        return {"n_dims": nd.value, "dims": [dims[i] for i in range(nd.value)], "ggml_type": t.value, "offset": off.value}

    def read_tensor_data(self, name) -> bytes:
        L = lib()
        n = L.or_gguf_read_tensor_data(self.h, name.encode(), None, 0)
        if n == 0:
            return b""
        buf = np.zeros(n, dtype=np.uint8)
        L.or_gguf_read_tensor_data(self.h, name.encode(), buf.ctypes.data_as(C.POINTER(C.c_uint8)), n)
        return buf.tobytes()

    def metadata_u64(self, key):
        v = C.c_uint64()
        return v.value if lib().or_gguf_meta_u64(self.h, key.encode(), C.byref(v)) else None

    def metadata_i64(self, key):
        v = C.c_int64()
        return v.value if lib().or_gguf_meta_i64(self.h, key.encode(), C.byref(v)) else None

    def metadata_f32(self, key):
        v = C.c_float()
        return v.value if lib().or_gguf_meta_f32(self.h, key.encode(), C.byref(v)) else None

    def metadata_bool(self, key):
        v = C.c_int()
        return bool(v.value) if lib().or_gguf_meta_bool(self.h, key.encode(), C.byref(v)) else None

    def metadata_string(self, key):
        buf = C.create_string_buffer(4096)
        return buf.value.decode() if lib().or_gguf_meta_string(self.h, key.encode(), buf, 4096) else None

    def vocab_size(self):
        v = C.c_uint64()
        return v.value if lib().or_gguf_vocab_size(self.h, C.byref(v)) else None

    def config(self):
        c = _Cfg()
        err = C.create_string_buffer(512)
        if lib().or_config_from_gguf(self.h, C.byref(c), err, 512):
            raise ValueError(err.value.decode())
        return {f: getattr(c, f) for f, _ in _Cfg._fields_}


def n_ff(n_embd, mult):
    return lib().or_config_n_ff(n_embd, mult)


# ---------------- model ----------------
class Model:
    def __init__(self, path: str, resident: bool = False, threads: int | None = None):
        err = C.create_string_buffer(512)
        self.h = lib().or_model_load(path.encode(), 1 if resident else 0, err, 512)
        if not self.h:
            raise ValueError(err.value.decode())
        c = _Cfg()
        lib().or_model_config(self.h, C.byref(c))
        self.cfg = {f: getattr(c, f) for f, _ in _Cfg._fields_}
        self.set_threads(threads or os.cpu_count() or 1)

    def set_threads(self, n):
        lib().or_model_set_threads(self.h, int(n))

    def close(self):
        if self.h:
            lib().or_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def time_layer(self, layer=0):
        """(seconds, macs) of one token's matmuls of `layer` in reference i-j-p order."""
        macs = C.c_double()
        s = lib().or_time_layer(self.h, layer, C.byref(macs))
        return s, macs.value

    def time_token(self, kv, token, pos, layers=0):
        """One decode token in the reference's order and data movement, one
        thread (or_time_token): (seconds in the first `layers` layers (0: all),
        seconds in the output head and greedy pick, picked id)."""
        out = (C.c_double * 2)()
        tok = lib().or_time_token(self.h, kv.h, int(token), int(pos), int(layers), out)
        if tok < 0:
            raise ValueError("or_time_token: cache full or token out of range")
        return out[0], out[1], int(tok)

    def kv(self, max_ctx, kv_f16=False):
        return KV(self, max_ctx, kv_f16)

    def forward(self, tokens, pos, kv, algo=1, hidden=False):
        t, tp = _u32(tokens)
        V, d, L = self.cfg["vocab_size"], self.cfg["n_embd"], self.cfg["n_layers"]
        logits = np.zeros(t.size * V, dtype=np.float32)
        hid = np.zeros(L * t.size * d, dtype=np.float32) if hidden else None
        rc = lib().or_forward(self.h, tp, t.size, pos, kv.h, logits.ctypes.data_as(C.POINTER(C.c_float)),
                              hid.ctypes.data_as(C.POINTER(C.c_float)) if hidden else None, algo)
        if rc:
            raise ValueError(f"or_forward failed: {rc}")
        return (logits, hid.reshape(L, t.size, d)) if hidden else logits

    def prefill(self, tokens, pos0, kv, logits=True, hidden=False):
        t, tp = _u32(tokens)
        V, d, L = self.cfg["vocab_size"], self.cfg["n_embd"], self.cfg["n_layers"]
        lg = np.zeros(V, dtype=np.float32) if logits else None
        hid = np.zeros(L * t.size * d, dtype=np.float32) if hidden else None
        rc = lib().or_prefill(self.h, tp, t.size, pos0, kv.h,
                              lg.ctypes.data_as(C.POINTER(C.c_float)) if logits else None,
                              hid.ctypes.data_as(C.POINTER(C.c_float)) if hidden else None)
        if rc:
            raise ValueError(f"or_prefill failed: {rc}")
        return lg, (hid.reshape(L, t.size, d) if hidden else None)

    def generate(self, prompt, max_tokens, temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=1.0,
                 stop_ids=(), seed=0, fast=True, kv_f16=False):
        p, pp = _u32(prompt)
        st, sp = _u32(np.array(stop_ids, dtype=np.uint32) if len(stop_ids) else np.zeros(1, dtype=np.uint32))
        g = _GenCfg(max_tokens, temperature, top_k, top_p, repetition_penalty, sp, len(stop_ids), seed, 1 if fast else 0)
        out = np.zeros(max(max_tokens, 1), dtype=np.uint32)
        n = lib().or_generate(self.h, C.byref(g), pp, p.size, out.ctypes.data_as(C.POINTER(C.c_uint32)), out.size,
                              1 if kv_f16 else 0)
        if n < 0:
            raise ValueError("or_generate failed")
        return out[:n].copy()


class KV:
    def __init__(self, model: Model, max_ctx: int, kv_f16: bool = False):
        self.model = model
        self.h = lib().or_kv_new(model.h, max_ctx, 1 if kv_f16 else 0)
        self.kvd = model.cfg["n_kv_heads"] * model.cfg["head_dim"]

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_kv_free(self.h)
            self.h = None

    def __len__(self):
        return lib().or_kv_len(self.h)

    def set(self, layer, k, v):
        """layer `layer` rows from k, v ([len][n_kv*hd] f32); the cache length
        becomes len"""
        k, kp = _f(np.asarray(k).reshape(-1))
        v, vp = _f(np.asarray(v).reshape(-1))
        if lib().or_kv_set(self.h, layer, kp, vp, k.size // self.kvd):
            raise IndexError("or_kv_set: bad layer or length")

    def fill_synthetic(self, length, seed=0):
        """timing only: `length` cached rows of pseudo-random K/V values"""
        lib().or_kv_fill_synthetic(self.h, int(length), int(seed))

    def clear(self):
        lib().or_kv_clear(self.h)

    def get(self, layer):
        n = len(self) * self.kvd
        k = np.zeros(max(n, 1), dtype=np.float32)
        v = np.zeros(max(n, 1), dtype=np.float32)
        if lib().or_kv_get(self.h, layer, k.ctypes.data_as(C.POINTER(C.c_float)), v.ctypes.data_as(C.POINTER(C.c_float))):
            raise IndexError(f"KV cache layer index out of range: {layer}")
        return k[:n], v[:n]


# ---------------- sampler ----------------
class Sampler:
    def __init__(self, temperature=0.7, top_k=40, top_p=0.95, repetition_penalty=1.15, frequency_penalty=0.0,
                 presence_penalty=0.0):
        self.cfg = _SamplerCfg(temperature, top_k, top_p, repetition_penalty, frequency_penalty, presence_penalty)
        self.h = lib().or_sampler_new(C.byref(self.cfg))

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_sampler_free(self.h)
            self.h = None

    def sample(self, logits, r: float = 0.5):
        l, lp = _f(logits)
        used = C.c_int()
        return lib().or_sampler_sample(self.h, lp, l.size, r, C.byref(used))

    def observe_token(self, tok):
        lib().or_sampler_observe(self.h, tok)

    def reset(self):
        lib().or_sampler_reset(self.h)

    def freq(self, tok):
        return lib().or_sampler_freq(self.h, tok)


def softmax(logits):
    l, lp = _f(logits)
    o = np.zeros(l.size, dtype=np.float32)
    lib().or_softmax_probs(lp, l.size, o.ctypes.data_as(C.POINTER(C.c_float)))
    return o


def top_k_filter(probs, k):
    p, pp = _f(probs)
    o = np.zeros(p.size, dtype=np.float32)
    lib().or_top_k_filter(pp, p.size, k, o.ctypes.data_as(C.POINTER(C.c_float)))
    return o


def top_p_filter(probs):
    p = np.array(probs, dtype=np.float32).copy()
    lib().or_top_p_filter(p.ctypes.data_as(C.POINTER(C.c_float)), p.size)
    return p


def categorical_sample(probs, r):
    p, pp = _f(probs)
    return lib().or_categorical_sample(pp, p.size, r)


def argmax(values):
    v, vp = _f(values)
    return lib().or_argmax(vp, v.size)
