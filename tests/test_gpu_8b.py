"""Greedy identity at full size: the 8B-shaped Q4_K_M synthetic model (Q6_K
attn_v / ffn_down / output head), a 2048-token uniform prompt, f32 KV cache.
The first 64 generated ids must equal the oracle's, committed as
tests/golden/8b_greedy.json by tests/golden/make_golden.py (the oracle needs
tens of minutes for this run, so the ids are a fixture rather than recomputed).
Generation follows GenerationState::generate (src/model.rs:638-705):
sequential prefill, re-feed of the last prompt token, greedy argmax."""
import hashlib
import json
import os

import pytest

from fishai_engine import synth
from fishai_engine.model import GenerationConfig, GenerationState, ModelWeights

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "8b_greedy.json")


def _digest(path, nbytes=1 << 24):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        h.update(f.read(nbytes))
    return h.hexdigest()


@pytest.mark.skipif(not os.path.exists(GOLDEN), reason="fixture not generated: python tests/golden/make_golden.py 8b")
@pytest.mark.parametrize("step_kernel", [False, True])
def test_8b_q4_k_m_first_64_greedy_ids_match_golden(step_kernel):
    g = json.load(open(GOLDEN))
    path = synth.cached_preset(g["preset"])
    # the synthetic file is the one the golden was made from
    assert _digest(path) == g["gguf_sha256_first16MiB"]
    m = ModelWeights.load_from_gguf(path, use_step_kernel=step_kernel)
    assert m.step_kernel_active == step_kernel
    try:
        prompt = g["prompt"]
        st = GenerationState(m, GenerationConfig(max_tokens=len(prompt) + len(g["greedy_ids"]), temperature=0.0,
                                                 top_k=0, top_p=1.0, repetition_penalty=1.0))
        ids = st.generate(prompt)
        assert len(ids) == 64
        assert ids == g["greedy_ids"]
    finally:
        m.close()


@pytest.mark.skipif(not os.path.exists(GOLDEN), reason="fixture not generated: python tests/golden/make_golden.py 8b")
@pytest.mark.parametrize("prefill", ["exact", "tc"])
def test_8b_benchmark_configuration_greedy_ids(prefill):
    """The configuration bench.py times: f16 KV cache, the prompt prefilled
    (exact = f32 token steps; tc = f16 tensor-core GEMMs and flash attention),
    the last prompt token fed again at position P (src/model.rs:656-657), then
    greedy steps through the captured decode graph.  The first 64 ids must
    equal the oracle's (whose cache is f32)."""
    from fishai_engine import _lib as L

    g = json.load(open(GOLDEN))
    path = synth.cached_preset(g["preset"])
    m = ModelWeights.load_from_gguf(path, use_tc_prefill=prefill == "tc")
    try:
        prompt = g["prompt"]
        kv = m.new_kv_cache(len(prompt) + 80, dtype=L.KV_F16)
        m.prefill(prompt, 0, kv, want_logits=False)
        ids = m.decode_greedy(kv, prompt[-1], len(prompt), 64).tolist()
        assert ids == g["greedy_ids"], [i for i in range(64) if ids[i] != g["greedy_ids"][i]][:1]
    finally:
        m.close()
