"""HTTP routes on the device model (src/http.rs:401-475, :603-766): load the
tiny model through /api/model/load, generate with temperature 0 and with
sampling, and check the ids against GenerationState on the same model and
seed; the SSE stream (new: the reference has no streaming route) must carry
the same ids; /api/sample must pick what the device Sampler picks."""
import json

import numpy as np
import pytest

pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402

from fishai_engine import synth  # noqa: E402
from fishai_engine.http import create_app  # noqa: E402
from fishai_engine.model import GenerationConfig, GenerationState, ModelWeights  # noqa: E402
from fishai_engine.sampling import Sampler, SamplerConfig  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def served():
    import os

    path = synth.cached_preset("tiny-q8_0")
    c = TestClient(create_app(model_dirs=[os.path.dirname(path)]))
    r = c.post("/api/model/load", json={"path": path})
    assert r.status_code == 200 and r.json()["success"], r.text
    m = ModelWeights.load_from_gguf(path)
    yield c, m
    m.close()


@pytest.mark.parametrize("temperature,seed", [(0.0, 0), (0.8, 7)])
def test_generate_and_stream_match_generation_state(served, temperature, seed):
    c, m = served
    prompt = "fish ai on B200"  # code points < vocab (32000)
    body = {"prompt": prompt, "max_tokens": len(prompt) + 24, "temperature": temperature, "top_k": 40,
            "top_p": 0.95, "repetition_penalty": 1.15, "seed": seed}
    r = c.post("/api/model/generate", json=body).json()
    cfg = GenerationConfig(max_tokens=body["max_tokens"], temperature=temperature, top_k=40, top_p=0.95,
                           repetition_penalty=1.15)
    want = GenerationState(m, cfg, seed=seed).generate([ord(ch) for ch in prompt])
    assert r["success"] and r["token_ids"] == want and r["n_generated_tokens"] == len(want) == 24
    assert r["n_prompt_tokens"] == len(prompt)
    events = [json.loads(line[6:]) for line in c.post("/api/model/generate/stream", json=body).text.splitlines()
              if line.startswith("data: ")]
    assert [e["token_id"] for e in events if "token_id" in e] == want
    assert events[-1]["done"] and events[-1]["n_generated_tokens"] == len(want)


def test_status_after_load(served):
    c, m = served
    s = c.get("/api/model/status").json()
    assert s["loaded"] and s["config"]["vocab_size"] == m.config.vocab_size
    assert c.get("/health").json()["model_loaded"] is True


def test_sample_route_matches_device_sampler(served):
    c, _ = served
    logits = np.random.default_rng(3).normal(0, 2, 5000).astype(np.float32)
    cfg = {"temperature": 0.7, "top_k": 40, "top_p": 0.9, "repetition_penalty": 1.2}
    freq = [0] * 5000
    freq[int(np.argmax(logits))] = 2
    r = c.post("/api/sample", json={"logits": logits.tolist(), "config": cfg, "token_freq": freq, "seed": 5})
    s = Sampler(SamplerConfig(0.7, 40, 0.9, 1.2, 0.0, 0.0), 5000, seed=5)
    for _ in range(2):
        s.observe_token(int(np.argmax(logits)))
    assert r.status_code == 200 and r.json()["token_id"] == s.sample(logits)
