"""Sampler — src/sampling.rs:14-310 on the device (Philox4x32-10 uniforms)."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L


@dataclass
class SamplerConfig:
    """src/sampling.rs:16-80"""
    temperature: float = 0.7
    top_k: int = 40
    top_p: float = 0.95
    repetition_penalty: float = 1.15
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0

    @staticmethod
    def greedy():
        return SamplerConfig(0.0, 0, 1.0, 1.0, 0.0, 0.0)

    @staticmethod
    def creative():
        return SamplerConfig(1.2, 80, 0.98, 1.05, 0.0, 0.0)

    @staticmethod
    def precise():
        return SamplerConfig(0.3, 20, 0.9, 1.3, 0.1, 0.1)

    def _c(self):
        return L.fa_sampler_config(self.temperature, self.top_k, self.top_p, self.repetition_penalty,
                                   self.frequency_penalty, self.presence_penalty)


class Sampler:
    """Sampler::new / sample / observe_token / reset (src/sampling.rs:95-165).
    Categorical draws use Philox4x32-10 keyed by `seed` with the sample index
    as counter (the reference uses the unseeded rand::rng())."""

    def __init__(self, config: SamplerConfig = None, vocab: int = 0, seed: int = 0, seeds=None):
        """seeds: one Philox key per sequence row (batched decode); else one row keyed by seed"""
        self.config = config or SamplerConfig()
        self.vocab = vocab
        keys = list(seeds) if seeds is not None else [seed]
        self.n_seq = len(keys)
        arr = (C.c_uint64 * self.n_seq)(*keys)
        h = C.c_void_p()
        L.check(L.lib().fa_sampler_create(C.byref(self.config._c()), self.n_seq, vocab, arr, C.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            L.lib().fa_sampler_free(h)
            self._h = None

    def sample(self, logits) -> int:
        a = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
        out = C.c_uint32()
        L.check(L.lib().fa_sample(self._h, 0, L.f32_ptr(a), a.size, C.byref(out)))
        return out.value

    def observe_token(self, token_id: int):
        L.check(L.lib().fa_sampler_observe(self._h, 0, token_id))

    def reset(self):
        L.check(L.lib().fa_sampler_reset(self._h, -1))

    def token_freq(self, token_id: int) -> int:
        """token_freq[token_id] (0 for ids never observed)"""
        c = C.c_uint32()
        L.check(L.lib().fa_sampler_freq(self._h, 0, token_id, C.byref(c)))
        return c.value
