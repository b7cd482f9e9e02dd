"""Device Sampler::sample (src/sampling.rs:110-152) against the oracle.

The reference draws its categorical uniform from rand::rng(); here both the
device and the oracle take r = Philox4x32-10(seed, sample index), so the ids
must be identical.  Known-answer cases follow the reference's own tests
(src/sampling.rs:317-501)."""
import os
import zlib

import numpy as np
import pytest

import oracle as O
from fishai_engine import _lib as L
from fishai_engine import synth
from fishai_engine.kv_cache import KVCache
from fishai_engine.model import GenerationConfig, GenerationState, ModelWeights
from fishai_engine.sampling import Sampler, SamplerConfig

pytestmark = pytest.mark.gpu


def _dev(cfg: SamplerConfig, vocab, seed=0):
    return Sampler(cfg, vocab, seed)


def _ora(cfg: SamplerConfig):
    return O.Sampler(cfg.temperature, cfg.top_k, cfg.top_p, cfg.repetition_penalty, cfg.frequency_penalty,
                     cfg.presence_penalty)


# ---- src/sampling.rs tests on the device sampler ----
def test_greedy_picks_max_logit():
    assert _dev(SamplerConfig.greedy(), 4).sample([0.1, 5.0, 0.3, 0.2]) == 1


def test_repetition_penalty_reduces_seen_tokens():
    s = _dev(SamplerConfig(0.0, 0, 1.0, 10.0, 0.0, 0.0), 2)
    s.observe_token(0)
    assert s.sample([5.0, 3.0]) == 1


def test_frequency_penalty():
    s = _dev(SamplerConfig(0.0, 0, 1.0, 1.0, 100.0, 0.0), 2)
    s.observe_token(0)
    s.observe_token(0)
    assert s.sample([200.0, 3.0]) == 1


def test_presence_penalty():
    s = _dev(SamplerConfig(0.0, 0, 1.0, 1.0, 0.0, 5.0), 2)
    s.observe_token(0)
    assert s.sample([4.0, 3.0]) == 1


def test_observe_and_reset():
    s = _dev(SamplerConfig(), 128)
    s.observe_token(42)
    s.observe_token(42)
    s.observe_token(100)
    assert s.token_freq(42) == 2 and s.token_freq(100) == 1 and s.token_freq(7) == 0
    s.reset()
    assert s.token_freq(42) == 0 and s.token_freq(100) == 0


def test_default_config_prefers_dominant_token():
    logits = np.zeros(768, np.float32)
    logits[100], logits[200], logits[300] = 10.0, 8.0, 6.0
    s = _dev(SamplerConfig(), 768, seed=3)
    counts = np.zeros(768, int)
    for _ in range(100):
        counts[s.sample(logits)] += 1
    assert counts[100] > 50


def test_categorical_certain_token():
    # probabilities exactly (0, 0, 1, 0)
    s = _dev(SamplerConfig(1.0, 0, 1.0, 1.0, 0.0, 0.0), 4)
    for _ in range(20):
        assert s.sample([-np.inf, -np.inf, 0.0, -np.inf]) == 2


def test_empty_logits_give_zero():
    assert _dev(SamplerConfig(), 8).sample(np.zeros(0, np.float32)) == 0


# ---- seeded parity with the oracle ----
CONFIGS = {
    "greedy": SamplerConfig.greedy(),
    "default": SamplerConfig(),
    "creative": SamplerConfig.creative(),
    "precise": SamplerConfig.precise(),
    "t1_nofilter": SamplerConfig(1.0, 0, 1.0, 1.0, 0.0, 0.0),
    "top_p_only": SamplerConfig(0.9, 0, 0.9, 1.1, 0.0, 0.0),          # whole-row sort
    "top_k_large": SamplerConfig(1.3, 3000, 0.97, 1.0, 0.05, 0.02),   # whole-row sort, k above the fast path
    "greedy_top_p": SamplerConfig(0.0, 40, 0.9, 1.0, 0.0, 0.0),
}


def _logits(kind, V, rng):
    if kind == "flat":
        return rng.normal(0.0, 1.0, V).astype(np.float32)
    if kind == "peaked":
        x = rng.normal(0.0, 2.0, V).astype(np.float32)
        x[rng.integers(0, V, 5)] += 12.0
        return x
    if kind == "ties":  # many equal values: top-k / sort tie-breaking by index
        return rng.integers(-3, 4, V).astype(np.float32)
    if kind == "dominant":  # one token above 0.999: top-p zeroes everything -> token 0
        x = rng.normal(0.0, 0.5, V).astype(np.float32)
        x[V // 3] = 40.0
        return x
    raise ValueError(kind)


@pytest.mark.parametrize("cfg_name", list(CONFIGS))
@pytest.mark.parametrize("kind", ["flat", "peaked", "ties", "dominant"])
def test_sampler_matches_oracle(cfg_name, kind):
    cfg = CONFIGS[cfg_name]
    V = 32000 if kind != "ties" else 5000
    rng = np.random.default_rng(zlib.crc32(f"{cfg_name}/{kind}".encode()))
    seed = 1000 + len(cfg_name)
    dev, ora = _dev(cfg, V, seed), _ora(cfg)
    n_samples = 24
    for i in range(n_samples):
        lg = _logits(kind, V, rng)
        a = dev.sample(lg)
        b = ora.sample(lg, O.philox_uniform(seed, i))
        assert a == b, (i, a, b)
        dev.observe_token(a)
        ora.observe_token(b)
    if kind == "dominant" and 0.0 < cfg.top_p < 1.0:
        assert a == 0  # the reference's 0.999 cut removes the dominant token itself


def test_sampler_full_vocab_matches_oracle():
    cfg = SamplerConfig(0.8, 40, 0.9, 1.15, 0.0, 0.0)
    V = 128256
    rng = np.random.default_rng(11)
    dev, ora = _dev(cfg, V, 1000), _ora(cfg)
    for i in range(12):
        lg = rng.normal(0.0, 1.5, V).astype(np.float32)
        a, b = dev.sample(lg), ora.sample(lg, O.philox_uniform(1000, i))
        assert a == b, i
        dev.observe_token(a)
        ora.observe_token(b)


def test_sample_device_rows():
    """fa_sample_device: several sequences, each its own seed and counter."""
    import ctypes as C

    import torch

    cfg = SamplerConfig(0.8, 40, 0.9, 1.0, 0.0, 0.0)
    n_seq, V = 4, 4096
    seeds = (C.c_uint64 * n_seq)(*[1000 + i for i in range(n_seq)])
    h = C.c_void_p()
    L.check(L.lib().fa_sampler_create(C.byref(cfg._c()), n_seq, V, seeds, C.byref(h)))
    try:
        rng = np.random.default_rng(5)
        oras = [_ora(cfg) for _ in range(n_seq)]
        for step in range(6):
            lg = rng.normal(0.0, 1.0, (n_seq, V)).astype(np.float32)
            t = torch.from_numpy(lg).cuda()
            ids = np.zeros(n_seq, np.uint32)
            L.check(L.lib().fa_sample_device(h, C.c_void_p(t.data_ptr()), n_seq, None,
                                             ids.ctypes.data_as(C.POINTER(C.c_uint32)), None))
            want = [oras[i].sample(lg[i], O.philox_uniform(1000 + i, step)) for i in range(n_seq)]
            assert ids.tolist() == want, step
    finally:
        L.lib().fa_sampler_free(h)


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    return synth.write_preset("tiny-q8_0", str(tmp_path_factory.mktemp("smp") / "tiny.gguf"))


@pytest.mark.parametrize("step_kernel", [False, True])
def test_sampled_generate_matches_oracle(tiny, step_kernel):
    """GenerationState::generate with T 0.8, k 40, p 0.9, rep 1.15: the sampler
    runs on the device after every step; ids equal the oracle's."""
    dev = ModelWeights.load_from_gguf(tiny, use_step_kernel=step_kernel)
    ref = O.Model(tiny, threads=os.cpu_count() or 4)
    prompt = np.random.default_rng(2).integers(3, 32000, 24).tolist()
    gc = GenerationConfig(max_tokens=24 + 64, temperature=0.8, top_k=40, top_p=0.9, repetition_penalty=1.15)
    for seed in (7, 1000):
        got = GenerationState(dev, gc, seed=seed).generate(prompt)
        want = ref.generate(prompt, gc.max_tokens, temperature=0.8, top_k=40, top_p=0.9, repetition_penalty=1.15,
                            seed=seed, fast=True).tolist()
        assert got == want, seed
    dev.close()


def test_generate_step_loop_matches_oracle(tiny):
    """generate_step (forward, device Sampler::sample, observe) driven from the host, teacher-forced:
    each step's logits match the oracle's forward of the same token within the f32 bar, and each id
    equals the oracle sampler applied to the device's logits with the same Philox uniform and observe
    history.  (Comparing against a whole oracle generation instead would turn an f32 rounding
    difference in the logits into a different draw whenever a uniform lands next to a boundary of
    the categorical walk, which near-uniform logits make likely.)"""
    dev = ModelWeights.load_from_gguf(tiny)
    ref = O.Model(tiny, threads=os.cpu_count() or 4)
    prompt = [17, 4242, 9, 31000, 77]
    gc = GenerationConfig(max_tokens=len(prompt) + 20, temperature=1.1, top_k=0, top_p=0.95, repetition_penalty=1.3)
    st = GenerationState(dev, gc, seed=21)
    st.kv_cache = KVCache(dev, gc.max_tokens + 1, 1, L.KV_F32)
    for i, t in enumerate(prompt):  # prefill, as generate() does
        dev.forward([t], i, st.kv_cache)
    st.token_ids, st.pos = list(prompt), len(prompt)
    seen, fwd = [], dev.forward

    def recording_forward(tokens, pos, kv):
        lg = fwd(tokens, pos, kv)
        seen.append((list(tokens), pos, np.array(lg, dtype=np.float32).reshape(-1)))
        return lg

    dev.forward = recording_forward
    got, last = [], prompt[-1]
    while True:
        nxt = st.generate_step(last)
        if nxt is None:
            break
        got.append(nxt)
        last = nxt
    assert len(got) == gc.max_tokens - len(prompt)
    kr = ref.kv(gc.max_tokens + 1)
    ref.prefill(prompt, 0, kr)
    ora = O.Sampler(1.1, 0, 0.95, 1.3, 0.0, 0.0)
    for s, (toks, pos, lg) in enumerate(seen):
        lr = np.asarray(ref.forward(toks, pos, kr, algo=1)).reshape(-1)
        assert np.max(np.abs(lg - lr)) / np.max(np.abs(lr)) <= 1e-4, s
        want = ora.sample(lg, O.philox_uniform(21, s))
        assert got[s] == want, s
        ora.observe_token(want)
    dev.close()
