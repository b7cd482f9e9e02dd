"""Full-shape checks of the kernels behind the benchmark figures, on
one-layer models with the benchmark's widths (Llama-3-8B shape: d 4096,
32 query / 8 KV heads, head_dim 128, FFN 14336, vocab 128256):

* the tcgen05 token GEMM (prefill and batched decode) at the down
  projection (K = 14336) and the output head (N = 128256, 1002 column tiles
  of stream-K work) for 64 and 2048 tokens, against f16(X) . f16(W) summed
  in f32 by the host BLAS (the reference's matmul is src/tensor.rs:244-258);
  bar 1e-3 of max |Y|;
* batch-1 decode attention (k_attn_paged) over 2048+ cached positions of the
  f16 paged cache, against the oracle with the same f16-rounded cache
  (src/tensor.rs:451-551; the f32 path keeps the 1e-4 bar);
* batched decode (k_attn_decode_rows: 64 rows over 4096+ positions, each
  (row, kv head) split 3 ways) against the oracle forward on the same cache
  contents, 1e-2 (the f16 tensor-core bar)."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
from fishai_engine import _lib as L
from fishai_engine import synth
from fishai_engine.model import ModelWeights

pytestmark = pytest.mark.gpu


def mar(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _w(g, name):
    i = g.tensor_info(name)
    ne0, ne1 = (i["dims"] + [1])[:2]
    return O.dequantize(g.read_tensor_data(name), i["ggml_type"], ne0 * ne1).reshape(ne1, ne0)


def _f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def _gemm(dev, proj, layer, x):
    T, n = x.shape[0], C.c_uint32()
    L.check(L.lib().fa_gemm_tokens(dev._h, proj, layer, L.f32_ptr(x), T, None, C.byref(n)))
    y = np.zeros((T, n.value), np.float32)
    L.check(L.lib().fa_gemm_tokens(dev._h, proj, layer, L.f32_ptr(x), T, L.f32_ptr(y), C.byref(n)))
    return y


@pytest.fixture(scope="module")
def q4km_1layer():
    path = synth.cached_preset("llama3-8b-q4_k_m", n_layers=1)
    dev = ModelWeights.load_from_gguf(path, use_tc_prefill=True)
    yield path, dev
    dev.close()


@pytest.mark.parametrize("proj,name", [(3, "blk.0.ffn_down.weight"), (4, "output.weight")])
@pytest.mark.parametrize("T", [64, 2048])
def test_token_gemm_at_benchmark_shapes(q4km_1layer, proj, name, T):
    path, dev = q4km_1layer
    g = O.GGUF(path)
    W = _f16(_w(g, name))
    x = np.random.default_rng(proj * 7 + T).normal(0.0, 1.0, (T, W.shape[0])).astype(np.float32)
    y = _gemm(dev, proj, 0, x)
    assert y.shape == (T, W.shape[1])
    ref = _f16(x) @ W
    assert np.isfinite(y).all()
    assert mar(y, ref) <= 1e-3


def test_paged_decode_attention_f16_cache_2048_positions(q4km_1layer):
    """2048-token prompt fed by the f32 token steps into the f16 cache, then
    one decode step at position 2048.  The attention is checked on identical
    cache contents: the oracle's cache is loaded with the device's f16 entries
    (widened exactly), so only f32 arithmetic differs and the 1e-4 bar holds.
    The prefilled entries themselves are checked against the oracle's own
    f16-rounded prefill at the f16 bar (two f32 paths that differ by ~1e-6
    round a few entries to neighbouring f16 values)."""
    path, dev = q4km_1layer
    dev.set_tc_prefill(False)
    try:
        P = 2048
        prompt = np.random.default_rng(5).integers(3, dev.config.vocab_size, P).tolist()
        kv = dev.new_kv_cache(P + 8, dtype=L.KV_F16)
        dev.prefill(prompt, 0, kv, want_logits=False)
        kd, vd = kv.get(0)
        got = dev.forward([prompt[-1]], P, kv)
        ref = O.Model(path, threads=os.cpu_count() or 8)
        kr = ref.kv(P + 8, kv_f16=True)
        kr.set(0, kd, vd)
        want = ref.forward([prompt[-1]], P, kr, algo=1)
        assert mar(got, want) <= 1e-4
        kp = ref.kv(P + 8, kv_f16=True)
        ref.prefill(prompt, 0, kp, logits=False)
        kw, vw = kp.get(0)
        assert mar(kd, kw) <= 1e-2 and mar(vd, vw) <= 1e-2
    finally:
        dev.set_tc_prefill(True)


def test_batched_decode_64_rows_4096_positions():
    """64 sequences of 4096 cached positions (tensor-core prefill, f16 cache),
    one batched step (attention split 3 ways per row and kv head): rows 0, 31
    and 63 against the oracle forward on the same cache contents."""
    from fishai_engine.sampling import Sampler, SamplerConfig

    path = synth.cached_preset("llama3-8b-q8_0", n_layers=1)
    dev = ModelWeights.load_from_gguf(path, use_tc_prefill=True)
    try:
        B, P = 64, 4096
        V = dev.config.vocab_size
        kv = dev.new_kv_cache(P + 16, dtype=L.KV_F16, n_seq=B)
        rng = np.random.default_rng(11)
        last = []
        for r in range(B):
            pr = rng.integers(3, V, P).tolist()
            dev.prefill(pr, 0, kv, seq=r, want_logits=False)
            last.append(pr[-1])
        smp = Sampler(SamplerConfig(0.0, 0, 1.0, 1.0, 0.0, 0.0), V, seeds=list(range(B)))
        ids, lg = dev.decode_batch(kv, last, [P] * B, smp, 1, want_logits=True)
        ref = O.Model(path, threads=os.cpu_count() or 8)
        for r in (0, 31, 63):
            k, v = kv.get(0, seq=r)
            kr = ref.kv(P + 8)
            kr.set(0, k[:P * 1024], v[:P * 1024])
            want = ref.forward([last[r]], P, kr, algo=1)
            assert mar(lg[0, r], want) <= 1e-2, r
            assert int(ids[0, r]) == int(np.argmax(lg[0, r]))
    finally:
        dev.close()
