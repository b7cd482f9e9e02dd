"""Generates the committed golden fixtures with the oracle (the C
restatement of the reference CPU path, fast bit-identical mode) on the
seeded synthetic GGUF files written by fishai_engine.synth.

  python tests/golden/make_golden.py tiny     # tiny Q8_0: 32-token prompt, 128 greedy ids
  python tests/golden/make_golden.py 8b       # 8B Q4_K_M: 2048-token prompt, 64 greedy ids
  python tests/golden/make_golden.py 7b       # 7B Q4_0 (Q6_K head), MHA: 512-token prompt, 64 greedy ids
  python tests/golden/make_golden.py 70b2     # 70B-shaped Q4_K, first 2 of 80 layers: 64-token prompt, 16 ids

Prompts are uniform ids in [3, vocab) from numpy default_rng(seed of the
config).  Greedy = GenerationState::generate with SamplerConfig::greedy()
(temperature 0, no penalties), including the re-feed of the last prompt
token (src/model.rs:638-705)."""
import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "fishai-engine_b200"), os.path.join(ROOT, "oracle")]

import oracle as O  # noqa: E402
from fishai_engine import synth  # noqa: E402

CASES = {
    "tiny": dict(preset="tiny-q8_0", seed=0, prompt=32, gen=128),
    "8b": dict(preset="llama3-8b-q4_k_m", seed=2, prompt=2048, gen=64),
    "7b": dict(preset="llama2-7b-q4_0", seed=1, prompt=512, gen=64),
    # full-width 70B layers (d 8192, 64/8 heads, FFN 28672) at reduced depth:
    # the tensor-parallel shards are checked against these ids
    "70b2": dict(preset="llama3-70b-q4_k", seed=4, prompt=64, gen=16, override=dict(n_layers=2)),
}


def file_digest(path, nbytes=1 << 24):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        h.update(f.read(nbytes))
    return h.hexdigest()


def make(name):
    c = CASES[name]
    override = c.get("override", {})
    path = synth.cached_preset(c["preset"], **override)
    m = O.Model(path, threads=os.cpu_count() or 8)
    V = m.cfg["vocab_size"]
    prompt = np.random.default_rng(c["seed"]).integers(3, V, c["prompt"]).tolist()
    t0 = time.time()
    kv = m.kv(c["prompt"] + 8)
    last, _ = m.prefill(prompt, 0, kv)  # logits of the last prompt token (discarded by generate)
    ids = m.generate(prompt, c["prompt"] + c["gen"], fast=True).tolist()
    out = {
        "preset": c["preset"], "override": override, "seed": c["seed"], "prompt_len": c["prompt"], "prompt": prompt,
        "greedy_ids": ids, "gguf_sha256_first16MiB": file_digest(path),
        "prefill_last_logits_top8": np.argsort(-last)[:8].tolist(),
        "prefill_last_logits_sum": float(np.sum(last.astype(np.float64))),
        "seconds": time.time() - t0,
    }
    with open(os.path.join(HERE, f"{name}_greedy.json"), "w") as f:
        json.dump(out, f)
    print(name, "done in", out["seconds"], "s")


if __name__ == "__main__":
    for n in sys.argv[1:] or ["tiny"]:
        make(n)
