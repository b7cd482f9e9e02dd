"""ModelConfig / ModelWeights / GenerationConfig / GenerationState —
src/model.rs:35-716, with the forward pass on the device."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

from . import _lib as L
from .gguf import GGUFFile
from .kv_cache import KVCache
from .sampling import Sampler, SamplerConfig


@dataclass
class ModelConfig:
    """src/model.rs:37-60"""
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    n_embd: int
    vocab_size: int
    context_len: int
    ffn_dim_multiplier: float
    norm_eps: float
    rope_base: float
    rope_freq_dim: int
    n_ff_used: int = 0
    tied_output: bool = False

    def n_ff(self) -> int:
        """src/model.rs:66-70: roundup256(int(n_embd * ffn_dim_multiplier))"""
        return L.lib().fa_config_n_ff(self.n_embd, self.ffn_dim_multiplier)

    def n_head_dim(self) -> int:
        return self.head_dim

    def head_count_kv(self) -> int:
        return self.n_kv_heads

    @classmethod
    def _from_c(cls, c: L.fa_config) -> "ModelConfig":
        return cls(c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.n_embd, c.vocab_size, c.context_len,
                   c.ffn_dim_multiplier, c.norm_eps, c.rope_base, c.rope_freq_dim, c.n_ff_used, bool(c.tied_output))

    @classmethod
    def from_gguf(cls, gguf: GGUFFile) -> "ModelConfig":
        """ModelConfig::from_gguf (src/model.rs:92-180)"""
        c = L.fa_config()
        L.check(L.lib().fa_config_from_gguf(gguf._h, C.byref(c)))
        return cls._from_c(c)


class ModelWeights:
    """Weights resident on one B200 (native GGML blocks re-laid per column
    chunk).  load_from_gguf mirrors src/model.rs:252-298."""

    def __init__(self, handle, config: ModelConfig):
        self._h = handle
        self.config = config
        r, w = C.c_int(), C.c_int()
        hl, kvl, fl = C.c_uint32(), C.c_uint32(), C.c_uint32()
        L.check(L.lib().fa_model_tp(handle, C.byref(r), C.byref(w), C.byref(hl), C.byref(kvl), C.byref(fl)))
        self.tp_rank, self.tp_world = r.value, w.value
        self.local_heads, self.local_kv_heads, self.local_ff = hl.value, kvl.value, fl.value

    @classmethod
    def load_from_gguf(cls, gguf, config: Optional[ModelConfig] = None, device: int = 0, use_graphs: bool = True,
                       use_pdl: bool = True, use_step_kernel: bool = False, use_tc_prefill: bool = False,
                       tp_rank: int = 0, tp_world: int = 1, nccl_id: Optional[bytes] = None) -> "ModelWeights":
        """tp_world > 1: this process's rank of a tensor-parallel model (one
        process per GPU); nccl_id = tp_unique_id() made on rank 0 and shared
        with every rank.  All ranks must then make the same calls."""
        path = gguf.path if isinstance(gguf, GGUFFile) else str(gguf)
        o = L.fa_model_opts()
        L.lib().fa_model_opts_default(C.byref(o))
        o.device, o.use_graphs, o.use_pdl = device, int(use_graphs), int(use_pdl)
        o.use_step_kernel = int(use_step_kernel)
        o.use_tc_prefill = int(use_tc_prefill)
        o.tp_rank, o.tp_world = tp_rank, tp_world
        uid = None
        if tp_world > 1:
            if nccl_id is None or len(nccl_id) != 128:
                raise ValueError("tensor parallelism needs the 128-byte id from tp_unique_id() on rank 0")
            uid = C.create_string_buffer(bytes(nccl_id), 128)
            o.nccl_id = C.cast(uid, C.c_void_p)
        h = C.c_void_p()
        L.check(L.lib().fa_model_load(path.encode(), C.byref(o), C.byref(h)))
        c = L.fa_config()
        L.check(L.lib().fa_model_config(h, C.byref(c)))
        return cls(h, ModelConfig._from_c(c))

    def set_tc_prefill(self, on: bool):
        """prefill() on the f16 tensor-core path (True) or the f32 token steps"""
        L.check(L.lib().fa_model_set_tc_prefill(self._h, int(on)))

    def step_launches(self) -> int:
        """kernel launches in one replay of the captured decode step (0 before
        the first decode)"""
        n = C.c_uint32()
        L.check(L.lib().fa_model_step_launches(self._h, C.byref(n)))
        return n.value

    @property
    def step_kernel_active(self) -> bool:
        """True when decode steps run as the persistent step kernel."""
        return bool(L.lib().fa_model_step_kernel_active(self._h))

    def close(self):
        if self._h:
            L.lib().fa_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def weight_bytes(self):
        dev, step = C.c_uint64(), C.c_uint64()
        L.check(L.lib().fa_model_weight_bytes(self._h, C.byref(dev), C.byref(step)))
        return dev.value, step.value

    def new_kv_cache(self, max_ctx: int = None, dtype: int = L.KV_F32, n_seq: int = 1) -> KVCache:
        return KVCache(self, max_ctx, n_seq, dtype)

    def forward(self, token_ids, pos: int, kv_cache: KVCache, seq: int = 0, return_argmax: bool = False,
                hidden: bool = False, want_logits: bool = True):
        """ModelWeights::forward (src/model.rs:316-455): logits [n * vocab];
        every token at `pos`, no mask, as in the reference.  want_logits=False
        leaves the logits on the device (None is returned in their place):
        only the argmax ids cross PCIe."""
        toks, tp = L.u32_array(token_ids)
        n, V = toks.size, self.config.vocab_size
        logits = np.zeros(n * V, dtype=np.float32) if want_logits else None
        am = np.zeros(n, dtype=np.uint32)
        hid = np.zeros(self.config.n_layers * n * self.config.n_embd, dtype=np.float32) if hidden else None
        L.check(L.lib().fa_forward(self._h, kv_cache._h, seq, tp, n, pos, L.f32_ptr(logits) if want_logits else None,
                                   am.ctypes.data_as(C.POINTER(C.c_uint32)), L.f32_ptr(hid) if hidden else None))
        out = [logits]
        if return_argmax:
            out.append(am)
        if hidden:
            out.append(hid.reshape(self.config.n_layers, n, self.config.n_embd))
        return out[0] if len(out) == 1 else tuple(out)

    def prefill(self, token_ids, start_pos: int, kv_cache: KVCache, seq: int = 0, want_logits: bool = True):
        """Causal prefill, equal to len(token_ids) single-token forwards."""
        toks, tp = L.u32_array(token_ids)
        logits = np.zeros(self.config.vocab_size, dtype=np.float32) if want_logits else None
        am = C.c_uint32()
        L.check(L.lib().fa_prefill(self._h, kv_cache._h, seq, tp, toks.size, start_pos,
                                   L.f32_ptr(logits) if want_logits else None, C.byref(am)))
        return logits, am.value

    def decode_batch(self, kv_cache: KVCache, tokens, positions, sampler, steps: int, want_logits: bool = False):
        """Sequences 0..b-1 advance `steps` tokens together (f16 tensor-core
        projections, per-row attention, device sampling).  Returns ids
        [steps][b] (and logits [steps][b][vocab] when asked)."""
        tk, tp = L.u32_array(tokens)
        ps, pp = L.u32_array(positions)
        b = tk.size
        ids = np.zeros((steps, b), dtype=np.uint32)
        lg = np.zeros((steps, b, self.config.vocab_size), dtype=np.float32) if want_logits else None
        L.check(L.lib().fa_decode_batch(self._h, kv_cache._h, b, tp, pp, sampler._h, steps,
                                        ids.ctypes.data_as(C.POINTER(C.c_uint32)),
                                        L.f32_ptr(lg) if want_logits else None))
        return (ids, lg) if want_logits else ids

    def decode_greedy(self, kv_cache: KVCache, first_token: int, pos: int, steps: int, seq: int = 0):
        ids = np.zeros(steps, dtype=np.uint32)
        L.check(L.lib().fa_decode_greedy(self._h, kv_cache._h, seq, first_token, pos, steps,
                                         ids.ctypes.data_as(C.POINTER(C.c_uint32))))
        return ids


def tp_unique_id() -> bytes:
    """a fresh NCCL unique id (rank 0 makes it; every rank passes it to
    ModelWeights.load_from_gguf)"""
    buf = C.create_string_buffer(128)
    L.check(L.lib().fa_tp_unique_id(buf))
    return buf.raw


@dataclass
class GenerationConfig:
    """src/model.rs:547-573"""
    max_tokens: int = 512
    temperature: float = 0.7
    top_k: int = 40
    top_p: float = 0.95
    repetition_penalty: float = 1.15
    stop_token_ids: List[int] = field(default_factory=list)


class GenerationState:
    """src/model.rs:581-716.  generate() runs the whole loop on the device
    (prefill, re-feed of the last prompt token, decode) with only token ids
    crossing PCIe."""

    def __init__(self, model: ModelWeights, config: GenerationConfig, seed: int = 0, kv_dtype: int = L.KV_F32):
        self.model = model
        self.config = config
        self.seed = seed
        self.kv_dtype = kv_dtype
        self.token_ids: List[int] = []
        self.pos = 0
        self.kv_cache = None
        self.sampler_config = SamplerConfig(config.temperature, config.top_k, config.top_p,
                                            config.repetition_penalty, 0.0, 0.0)
        self.sampler = None  # generate_step's Sampler (generate() runs its own on the device)

    def _gen_c(self):
        stops = np.asarray(self.config.stop_token_ids or [0], dtype=np.uint32)
        self._stops = stops
        return L.fa_gen_config(self.config.max_tokens, self.sampler_config._c(),
                               stops.ctypes.data_as(C.POINTER(C.c_uint32)), len(self.config.stop_token_ids),
                               self.seed, self.kv_dtype)

    def generate(self, prompt_tokens) -> List[int]:
        """src/model.rs:638-674"""
        p, pp = L.u32_array(prompt_tokens)
        g = self._gen_c()
        cap = max(self.config.max_tokens, 1)
        out = np.zeros(cap, dtype=np.uint32)
        n = C.c_uint32()
        L.check(L.lib().fa_generate(self.model._h, C.byref(g), pp, p.size, out.ctypes.data_as(C.POINTER(C.c_uint32)),
                                    cap, C.byref(n)))
        gen = out[: n.value].tolist()
        self.token_ids = list(p.tolist()) + gen
        self.pos = len(self.token_ids)
        return gen

    def generate_step(self, token_id: int) -> Optional[int]:
        """src/model.rs:681-705: forward, Sampler::sample on the device, observe"""
        if len(self.token_ids) >= self.config.max_tokens:
            return None
        if self.kv_cache is None:
            self.kv_cache = KVCache(self.model, max(self.config.max_tokens + 1, 16), 1, self.kv_dtype)
        if self.sampler is None:
            self.sampler = Sampler(self.sampler_config, self.model.config.vocab_size, self.seed)
        logits = self.model.forward([token_id], self.pos, self.kv_cache)
        nxt = self.sampler.sample(logits)
        self.sampler.observe_token(nxt)
        self.token_ids.append(nxt)
        self.pos += 1
        if nxt in self.config.stop_token_ids:
            return None
        return nxt

    def reset(self):
        """src/model.rs:710-715"""
        if self.kv_cache is not None:
            self.kv_cache.clear()
        if self.sampler is not None:
            self.sampler.reset()
        self.token_ids = []
        self.pos = 0
