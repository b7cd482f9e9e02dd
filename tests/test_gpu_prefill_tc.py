"""Tensor-core prefill (tcgen05 GEMMs, causal flash attention, f16 operands)
against the oracle's sequential f32 forwards: the 16-bit parity bar is
max-abs-rel 1e-2 on the last token's logits and on the cached K/V."""
import os

import numpy as np
import pytest

import oracle as O
from fishai_engine import _lib as L
from fishai_engine import synth
from fishai_engine.model import ModelWeights

pytestmark = pytest.mark.gpu
TOL_BF16 = 1e-2  # bf16/f16 accumulate bar


def max_abs_rel(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _spec(**kw):
    s = dict(n_layers=2, n_embd=512, n_heads=8, n_kv_heads=4, n_ff=1536, vocab=4096, context_len=4096,
             rope_base=500000.0, norm_eps=1e-5, sigma=0.02, type_embd=O.Q4_K, type_q=O.Q4_K, type_k=O.Q4_K,
             type_v=O.Q6_K, type_o=O.Q4_K, type_gate=O.Q4_K, type_up=O.Q4_K, type_down=O.Q6_K, type_out=O.Q6_K)
    s.update(kw)
    return s


MODELS = {
    "q8_0_hd64": None,
    "kq_hd64": _spec(),
    "kq_hd128": _spec(n_embd=1024, n_heads=8, n_kv_heads=2, n_ff=2816),
    "q4_0_mha": _spec(type_embd=O.Q4_0, type_q=O.Q4_0, type_k=O.Q4_0, type_v=O.Q4_0, type_o=O.Q4_0, type_gate=O.Q4_0,
                      type_up=O.Q4_0, type_down=O.Q4_0, type_out=O.Q6_K, n_kv_heads=8, rope_base=10000.0),
}


@pytest.fixture(scope="module", params=list(MODELS))
def pair(request, tmp_path_factory):
    path = str(tmp_path_factory.mktemp("ptc") / f"{request.param}.gguf")
    spec = MODELS[request.param]
    p = synth.write_preset("tiny-q8_0", path) if spec is None else synth.write(path, 13, **spec)
    dev = ModelWeights.load_from_gguf(p, use_tc_prefill=True)
    ref = O.Model(p, threads=os.cpu_count() or 4)
    yield dev, ref
    dev.close()


@pytest.mark.parametrize("kv_dtype", [L.KV_F16, L.KV_F32])
@pytest.mark.parametrize("n", [1, 45, 200])
def test_prefill_matches_oracle(pair, kv_dtype, n):
    dev, ref = pair
    V = dev.config.vocab_size
    toks = np.random.default_rng(n).integers(3, V, n).tolist()
    kd = dev.new_kv_cache(n + 8, dtype=kv_dtype)
    kr = ref.kv(n + 8, kv_f16=kv_dtype == L.KV_F16)
    lg, am = dev.prefill(toks, 0, kd)
    lr, _ = ref.prefill(toks, 0, kr)
    assert max_abs_rel(lg, lr) <= TOL_BF16
    assert am == int(np.argmax(lg))
    for layer in (0, dev.config.n_layers - 1):
        k_d, v_d = kd.get(layer)
        k_r, v_r = kr.get(layer)
        assert max_abs_rel(k_d, k_r) <= TOL_BF16 and max_abs_rel(v_d, v_r) <= TOL_BF16


def test_prefill_continues_a_cache(pair):
    """a second prefill appends after the cached positions (len0 > 0, start_pos > 0)"""
    dev, ref = pair
    V = dev.config.vocab_size
    toks = np.random.default_rng(7).integers(3, V, 250).tolist()
    kd, kr = dev.new_kv_cache(260), ref.kv(260)
    dev.prefill(toks[:100], 0, kd)
    lg, _ = dev.prefill(toks[100:], 100, kd)
    lr, _ = ref.prefill(toks, 0, kr)
    assert max_abs_rel(lg, lr) <= TOL_BF16


def test_prefill_crosses_the_chunk_size(tmp_path):
    """2100 tokens: two chunks (2048 + 52), the second attending to the first"""
    p = synth.write(str(tmp_path / "long.gguf"), 17, **_spec(n_layers=1, vocab=2048))
    dev = ModelWeights.load_from_gguf(p, use_tc_prefill=True)
    ref = O.Model(p, threads=os.cpu_count() or 4)
    toks = np.random.default_rng(3).integers(3, 2048, 2100).tolist()
    kd, kr = dev.new_kv_cache(2110), ref.kv(2110)
    lg, _ = dev.prefill(toks, 0, kd)
    lr, _ = ref.prefill(toks, 0, kr)
    assert max_abs_rel(lg, lr) <= TOL_BF16
    k_d, _ = kd.get(0)
    k_r, _ = kr.get(0)
    assert max_abs_rel(k_d, k_r) <= TOL_BF16
    dev.close()
