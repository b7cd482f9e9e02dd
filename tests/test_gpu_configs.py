"""Greedy identity for the other workload shapes bench.py reports at one GPU
(GenerationState::generate, src/model.rs:638-705: prefill, re-feed of the last
prompt token, greedy argmax), against goldens the oracle made
(tests/golden/make_golden.py):

* the Llama-2-7B shape, Q4_0 everywhere (the reference's high-nibble-first
  order, src/quant.rs:143-148) with a Q6_K output head, MHA (32/32 heads):
  512-token prompt, first 64 greedy ids, on the f32 path and on the
  benchmark's configuration (f16 KV cache, decode graph);
* the tiny Q8_0 shape in the benchmark's configuration (128 ids)."""
import hashlib
import json
import os

import pytest

from fishai_engine import _lib as L
from fishai_engine import synth
from fishai_engine.model import GenerationConfig, GenerationState, ModelWeights

pytestmark = pytest.mark.gpu

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _golden(name):
    p = os.path.join(HERE, name)
    if not os.path.exists(p):
        pytest.skip(f"fixture missing: {name}")
    return json.load(open(p))


def _digest(path, nbytes=1 << 24):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        h.update(f.read(nbytes))
    return h.hexdigest()


@pytest.fixture(scope="module")
def llama2_7b():
    g = _golden("7b_greedy.json")
    path = synth.cached_preset(g["preset"], **g.get("override", {}))
    assert _digest(path) == g["gguf_sha256_first16MiB"]
    m = ModelWeights.load_from_gguf(path)
    yield g, m
    m.close()


def test_7b_q4_0_generate_matches_golden(llama2_7b):
    g, m = llama2_7b
    prompt = g["prompt"]
    cfg = GenerationConfig(max_tokens=len(prompt) + 64, temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=1.0)
    assert GenerationState(m, cfg).generate(prompt) == g["greedy_ids"]


def test_7b_q4_0_benchmark_configuration_matches_golden(llama2_7b):
    g, m = llama2_7b
    prompt = g["prompt"]
    kv = m.new_kv_cache(len(prompt) + 80, dtype=L.KV_F16)
    m.prefill(prompt, 0, kv, want_logits=False)
    assert m.decode_greedy(kv, prompt[-1], len(prompt), 64).tolist() == g["greedy_ids"]


def test_tiny_benchmark_configuration_matches_golden():
    g = _golden("tiny_greedy.json")
    m = ModelWeights.load_from_gguf(synth.cached_preset(g["preset"]))
    try:
        prompt = g["prompt"]
        kv = m.new_kv_cache(len(prompt) + 140, dtype=L.KV_F16)
        m.prefill(prompt, 0, kv, want_logits=False)
        assert m.decode_greedy(kv, prompt[-1], len(prompt), 128).tolist() == g["greedy_ids"]
    finally:
        m.close()
