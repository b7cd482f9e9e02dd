"""Synthetic llama GGUF files for the five workload shapes (seeded N(0, sigma)
weights through fa_synth_write).  No dataset or checkpoint is involved."""
from __future__ import annotations

import ctypes as C
import os

from . import _lib as L

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = L.F32, L.F16, L.Q4_0, L.Q8_0, L.Q4_K, L.Q6_K

# name -> (spec fields, seed)
PRESETS = {
    # 4 layers, d 512, 8/2 heads, hd 64, FFN 1408, vocab 32000, ctx 512, Q8_0 everywhere
    "tiny-q8_0": (dict(n_layers=4, n_embd=512, n_heads=8, n_kv_heads=2, n_ff=1408, vocab=32000, context_len=512,
                       rope_base=10000.0, norm_eps=1e-5, sigma=0.02, type_embd=Q8_0, type_q=Q8_0, type_k=Q8_0,
                       type_v=Q8_0, type_o=Q8_0, type_gate=Q8_0, type_up=Q8_0, type_down=Q8_0, type_out=Q8_0), 0),
    # Llama-2-7B shape, Q4_0 with a Q6_K output head
    "llama2-7b-q4_0": (dict(n_layers=32, n_embd=4096, n_heads=32, n_kv_heads=32, n_ff=11008, vocab=32000,
                            context_len=4096, rope_base=10000.0, norm_eps=1e-5, sigma=0.02, type_embd=Q4_0,
                            type_q=Q4_0, type_k=Q4_0, type_v=Q4_0, type_o=Q4_0, type_gate=Q4_0, type_up=Q4_0,
                            type_down=Q4_0, type_out=Q6_K), 1),
    # Llama-3-8B shape, Q4_K_M mix: Q6_K for attn_v, ffn_down and the head
    "llama3-8b-q4_k_m": (dict(n_layers=32, n_embd=4096, n_heads=32, n_kv_heads=8, n_ff=14336, vocab=128256,
                              context_len=8192, rope_base=500000.0, norm_eps=1e-5, sigma=0.02, type_embd=Q4_K,
                              type_q=Q4_K, type_k=Q4_K, type_v=Q6_K, type_o=Q4_K, type_gate=Q4_K, type_up=Q4_K,
                              type_down=Q6_K, type_out=Q6_K), 2),
    # Llama-3-8B shape, Q8_0
    "llama3-8b-q8_0": (dict(n_layers=32, n_embd=4096, n_heads=32, n_kv_heads=8, n_ff=14336, vocab=128256,
                            context_len=8192, rope_base=500000.0, norm_eps=1e-5, sigma=0.02, type_embd=Q8_0,
                            type_q=Q8_0, type_k=Q8_0, type_v=Q8_0, type_o=Q8_0, type_gate=Q8_0, type_up=Q8_0,
                            type_down=Q8_0, type_out=Q8_0), 3),
    # Llama-3-70B shape, Q4_K with a Q6_K head
    "llama3-70b-q4_k": (dict(n_layers=80, n_embd=8192, n_heads=64, n_kv_heads=8, n_ff=28672, vocab=128256,
                             context_len=8192, rope_base=500000.0, norm_eps=1e-5, sigma=0.015, type_embd=Q4_K,
                             type_q=Q4_K, type_k=Q4_K, type_v=Q4_K, type_o=Q4_K, type_gate=Q4_K, type_up=Q4_K,
                             type_down=Q4_K, type_out=Q6_K), 4),
}


def write(path: str, seed: int, threads: int = 0, **fields) -> str:
    s = L.fa_synth_spec()
    s.threads = threads
    s.type_out = fields.pop("type_out", -1)
    for k, v in fields.items():
        setattr(s, k, v)
    L.check(L.lib().fa_synth_write(str(path).encode(), C.byref(s), seed))
    return str(path)


def preset_fields(name: str, **override):
    """(spec fields, seed) of a preset with some fields replaced"""
    fields, seed = PRESETS[name]
    f = dict(fields)
    f.update(override)
    seed = f.pop("seed", seed)
    return f, seed


def write_preset(name: str, path: str, threads: int = 0, writer=None, **override) -> str:
    """writer: a function with the signature of write() (default: this
    library's fa_synth_write)"""
    f, seed = preset_fields(name, **override)
    return (writer or write)(path, seed, threads, **f)


def cache_path(name: str, directory: str = None, **override) -> str:
    directory = directory or os.environ.get("FISHAI_SYNTH_DIR", "/tmp/fishai_synth")
    tag = "-".join(f"{k}{v}" for k, v in sorted(override.items()))
    return os.path.join(directory, f"{name}{'-' + tag if tag else ''}.gguf")


def cached_preset(name: str, directory: str = None, writer=None, **override) -> str:
    """Write the preset once into `directory` (default $FISHAI_SYNTH_DIR or
    /tmp/fishai_synth) and reuse it afterwards."""
    path = cache_path(name, directory, **override)
    os.makedirs(os.path.dirname(path), exist_ok=True)
    if not os.path.exists(path):
        tmp = f"{path}.tmp{os.getpid()}"
        write_preset(name, tmp, writer=writer, **override)
        os.replace(tmp, path)
    return path
