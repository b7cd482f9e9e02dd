"""ctypes binding of lib/libfishai_cuda.so (include/fishai_cuda.h).

The CUDA library is the only compute path: importing a module that needs it
raises if the library has not been built (no CPU fallback exists)."""
from __future__ import annotations

import ctypes as C
import os
import subprocess

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_ROOT, "lib", "libfishai_cuda.so")

OK = 0
ERR_INVALID, ERR_GGUF, ERR_UNSUPPORTED, ERR_OOM, ERR_CUDA, ERR_NCCL, ERR_CONTEXT, ERR_TIMEOUT = -1, -2, -3, -4, -5, -6, -7, -8

F32, F16, Q4_0, Q4_1, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 3, 6, 8, 12, 14
KV_F32, KV_F16 = 0, 1
DEBUG_WAIT_LIMIT_NS, DEBUG_WITHHOLD_WEIGHTS, DEBUG_FIXED_ORDER_SUMS = 1, 2, 3


class FishaiError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class fa_config(C.Structure):
    _fields_ = [
        ("n_layers", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
        ("n_embd", C.c_uint32), ("vocab_size", C.c_uint32), ("context_len", C.c_uint32),
        ("ffn_dim_multiplier", C.c_float), ("norm_eps", C.c_float), ("rope_base", C.c_float),
        ("rope_freq_dim", C.c_uint32), ("n_ff", C.c_uint32), ("n_ff_used", C.c_uint32), ("tied_output", C.c_int32),
    ]


class fa_model_opts(C.Structure):
    _fields_ = [("device", C.c_int32), ("use_graphs", C.c_int32), ("use_pdl", C.c_int32), ("tp_rank", C.c_int32),
                ("tp_world", C.c_int32), ("nccl_id", C.c_void_p), ("use_step_kernel", C.c_int32),
                ("use_tc_prefill", C.c_int32)]


class fa_sampler_config(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_uint32), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float), ("frequency_penalty", C.c_float), ("presence_penalty", C.c_float)]


class fa_gen_config(C.Structure):
    _fields_ = [("max_tokens", C.c_uint32), ("sampler", fa_sampler_config), ("stop_ids", C.POINTER(C.c_uint32)),
                ("n_stop", C.c_uint32), ("seed", C.c_uint64), ("kv_dtype", C.c_int32)]


class fa_synth_spec(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("n_embd", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
                ("n_ff", C.c_uint32), ("vocab", C.c_uint32), ("context_len", C.c_uint32), ("rope_base", C.c_float),
                ("norm_eps", C.c_float), ("sigma", C.c_float), ("type_embd", C.c_int32), ("type_q", C.c_int32),
                ("type_k", C.c_int32), ("type_v", C.c_int32), ("type_o", C.c_int32), ("type_gate", C.c_int32),
                ("type_up", C.c_int32), ("type_down", C.c_int32), ("type_out", C.c_int32), ("threads", C.c_uint32)]


# every entry point of include/fishai_cuda.h with its ctypes signature
_vp, _sz, _i, _u32, _u64, _f = C.c_void_p, C.c_size_t, C.c_int, C.c_uint32, C.c_uint64, C.c_float
_pu32, _pu64, _pf, _pi, _pi64 = C.POINTER(C.c_uint32), C.POINTER(C.c_uint64), C.POINTER(C.c_float), C.POINTER(C.c_int), C.POINTER(C.c_int64)
SIGNATURES = {
    "fa_last_error": ([C.c_char_p, _sz], _sz),
    "fa_version": ([], C.c_char_p),
    "fa_gguf_open": ([C.c_char_p, C.POINTER(_vp)], _i),
    "fa_gguf_close": ([_vp], None),
    "fa_gguf_version": ([_vp, _pu32], _i),
    "fa_gguf_alignment": ([_vp, _pu64], _i),
    "fa_gguf_tensor_count": ([_vp, C.POINTER(_sz)], _i),
    "fa_gguf_tensor_at": ([_vp, _sz, C.c_char_p, _sz, _pu32, _pu64, _pu32, _pu64], _i),
    "fa_gguf_tensor_info": ([_vp, C.c_char_p, _pu32, _pu64, _pu32, _pu64], _i),
    "fa_gguf_read_tensor_data": ([_vp, C.c_char_p, _vp, _sz, C.POINTER(_sz)], _i),
    "fa_gguf_meta_u64": ([_vp, C.c_char_p, _pu64, _pi], _i),
    "fa_gguf_meta_i64": ([_vp, C.c_char_p, _pi64, _pi], _i),
    "fa_gguf_meta_f32": ([_vp, C.c_char_p, _pf, _pi], _i),
    "fa_gguf_meta_bool": ([_vp, C.c_char_p, _pi, _pi], _i),
    "fa_gguf_meta_string": ([_vp, C.c_char_p, C.c_char_p, _sz, _pi], _i),
    "fa_gguf_vocab_size": ([_vp, _pu64, _pi], _i),
    "fa_config_from_gguf": ([_vp, C.POINTER(fa_config)], _i),
    "fa_config_n_ff": ([_u32, _f], _u32),
    "fa_dequantize": ([_i, _vp, _sz, _sz, _pf, C.POINTER(_sz)], _i),
    "fa_dequantize_device": ([_i, _vp, _sz, _sz, _vp, _vp], _i),
    "fa_model_opts_default": ([C.POINTER(fa_model_opts)], None),
    "fa_model_load": ([C.c_char_p, C.POINTER(fa_model_opts), C.POINTER(_vp)], _i),
    "fa_model_free": ([_vp], None),
    "fa_model_config": ([_vp, C.POINTER(fa_config)], _i),
    "fa_model_weight_bytes": ([_vp, _pu64, _pu64], _i),
    "fa_model_stream": ([_vp], _vp),
    "fa_model_step_kernel_active": ([_vp], _i),
    "fa_model_set_tc_prefill": ([_vp, C.c_int32], _i),
    "fa_model_step_launches": ([_vp, _pu32], _i),
    "fa_debug_set": ([_vp, C.c_int32, _u64], _i),
    "fa_model_tp": ([_vp, _pi, _pi, _pu32, _pu32, _pu32], _i),
    "fa_tp_unique_id": ([_vp], _i),
    "fa_tokenizer_create": ([C.POINTER(C.c_char_p), _u32, _pf, _u32, C.POINTER(C.c_int32), _u32, C.c_char_p, _vp,
                             C.POINTER(_vp)], _i),
    "fa_tokenizer_from_gguf": ([_vp, C.POINTER(_vp)], _i),
    "fa_tokenizer_free": ([_vp], None),
    "fa_tokenizer_encode": ([_vp, C.c_char_p, _sz, C.c_int32, C.c_int32, _pu32, _sz, C.POINTER(_sz)], _i),
    "fa_tokenizer_decode": ([_vp, _pu32, _sz, C.c_char_p, _sz, C.POINTER(_sz)], _i),
    "fa_tokenizer_info": ([_vp, _pu32, _vp], _i),
    "fa_tokenizer_piece": ([_vp, _u32, C.c_char_p, _sz, C.POINTER(_sz), C.POINTER(C.c_int32)], _i),
    "fa_tokenizer_byte_token": ([_vp, _u32, _pu32], _i),
    "fa_tokenizer_config_default": ([_vp], None),
    "fa_tp_shard": ([C.c_int32, _vp, _u32, _u32, C.c_int32, _u32, _u32, _vp, _sz, C.POINTER(_sz), _pu32], _i),
    "fa_kv_create": ([_vp, _u32, _u32, C.c_int32, C.POINTER(_vp)], _i),
    "fa_kv_free": ([_vp], None),
    "fa_kv_clear": ([_vp, C.c_int32], _i),
    "fa_kv_seq_len": ([_vp, _u32, _pu32], _i),
    "fa_kv_get": ([_vp, _u32, _u32, _pf, _pf], _i),
    "fa_forward": ([_vp, _vp, _u32, _pu32, _u32, _u32, _pf, _pu32, _pf], _i),
    "fa_prefill": ([_vp, _vp, _u32, _pu32, _u32, _u32, _pf, _pu32], _i),
    "fa_sampler_create": ([C.POINTER(fa_sampler_config), _u32, _u32, _pu64, C.POINTER(_vp)], _i),
    "fa_sampler_free": ([_vp], None),
    "fa_sample_device": ([_vp, _vp, _u32, _vp, _pu32, _vp], _i),
    "fa_sample": ([_vp, _u32, _pf, _u32, _pu32], _i),
    "fa_sampler_observe": ([_vp, _u32, _u32], _i),
    "fa_sampler_reset": ([_vp, C.c_int32], _i),
    "fa_sampler_freq": ([_vp, _u32, _u32, _pu32], _i),
    "fa_gemm_tokens": ([_vp, C.c_int32, _u32, _pf, _u32, _pf, _pu32], _i),
    "fa_profile_gemm": ([_vp, C.c_int32, _u32, _u32, _u32, _pf, C.POINTER(C.c_double)], _i),
    "fa_decode_batch": ([_vp, _vp, _u32, _pu32, _pu32, _vp, _u32, _pu32, _pf], _i),
    "fa_generate": ([_vp, C.POINTER(fa_gen_config), _pu32, _u32, _pu32, _u32, _pu32], _i),
    "fa_decode_greedy": ([_vp, _vp, _u32, _u32, _u32, _u32, _pu32], _i),
    "fa_profile_gemv": ([_vp, C.c_int32, _u32, _pf, _pu64], _i),
    "fa_sdpa": ([_vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp, _vp], _i),
    "fa_sdpa_noalloc": ([_vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp, _vp], _i),
    "fa_sdpa_host": ([_pf, _pf, _pf, _u32, _u32, _u32, _u32, _u32, _pf], _i),
    "fa_synth_write": ([C.c_char_p, C.POINTER(fa_synth_spec), _u64], _i),
}

_lib = None


def build() -> str:
    """Compile the library in-tree with its Makefile (nvcc, sm_100a)."""
    subprocess.run(["make", "-s", "-j8", "-C", _PKG_ROOT], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FishaiError(ERR_CUDA, f"CUDA library not built: {LIB_PATH} (run make in fishai-engine_b200)")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(2048)
    lib().fa_last_error(buf, 2048)
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != OK:
        raise FishaiError(rc, last_error())


def u32_array(seq):
    import numpy as np
    a = np.ascontiguousarray(np.asarray(seq, dtype=np.uint32))
    return a, a.ctypes.data_as(_pu32)


def f32_ptr(a):
    return a.ctypes.data_as(_pf)
