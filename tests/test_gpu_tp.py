"""Tensor parallelism on 2, 4 or 8 GPUs (one process per GPU, NCCL over
NVLink): every rank loads its shards, runs the same calls, and must produce
the reference's tokens.

* A small Q4_K model with 128-wide heads and two KV heads: at two ranks each
  rank's K/V shard is half of a 256-column super-block (re-encoded at load),
  the path eight-way parallelism takes on the 70B shape.  Logits of one
  forward against the oracle (1e-4, the f32 path) and 16 greedy ids from
  GenerationState::generate (src/model.rs:638-705) equal to the oracle's.
* The 70B shape at full width (d 8192, 64/8 heads, FFN 28672) with the
  first 2 of its 80 layers, on one GPU and tensor-parallel: 16 greedy ids
  equal to the committed golden, and the tensor-core prefill's last logits
  within 1e-2 of the oracle's.
Skipped when fewer GPUs are visible than the case needs."""
import json
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu

SMALL = dict(n_layers=2, n_embd=512, n_heads=4, n_kv_heads=2, n_ff=1024, vocab=2048, context_len=128,
             rope_base=500000.0, norm_eps=1e-5, sigma=0.015, type_embd=12, type_q=12, type_k=12, type_v=12,
             type_o=12, type_gate=12, type_up=12, type_down=12, type_out=14)


def _gpus():
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _worker(rank, world, uid, path, prompt, gen, q, tc):
    import sys

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    for p in (os.path.join(ROOT, "fishai-engine_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    from fishai_engine.model import GenerationConfig, GenerationState, ModelWeights

    out = {}
    try:
        m = ModelWeights.load_from_gguf(path, device=rank, tp_rank=rank, tp_world=world, nccl_id=uid,
                                        use_tc_prefill=tc)
        assert m.tp_world == world and m.tp_rank == rank
        kv = m.new_kv_cache(len(prompt) + gen + 8)
        out["logits"] = m.forward([prompt[0]], 0, kv)
        if tc:
            kv2 = m.new_kv_cache(len(prompt) + 8)
            out["prefill_logits"], _ = m.prefill(prompt, 0, kv2)
        cfg = GenerationConfig(max_tokens=len(prompt) + gen, temperature=0.0, top_k=0, top_p=1.0,
                               repetition_penalty=1.0)
        out["ids"] = GenerationState(m, cfg).generate(prompt)
        m.close()
    except Exception as e:  # reported to the parent, which fails the test
        out["error"] = repr(e)
    q.put((rank, out))


def _run(world, path, prompt, gen, tc=False):
    import multiprocessing as mp

    import sys

    sys.path.insert(0, os.path.join(ROOT, "fishai-engine_b200"))
    from fishai_engine.model import tp_unique_id

    uid = tp_unique_id() if world > 1 else None
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, uid, path, prompt, gen, q, tc)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in procs:
            r, out = q.get(timeout=600)
            res[r] = out
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.kill()
    for r in range(world):
        assert "error" not in res[r], res[r].get("error")
    return res


def _mar(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / np.max(np.abs(b)))


@pytest.mark.parametrize("world", [2])
def test_tp_half_superblock_kv_shards_match_oracle(world, tmp_path):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import sys

    sys.path.insert(0, os.path.join(ROOT, "fishai-engine_b200"))
    import oracle as O
    from fishai_engine import synth

    path = synth.write(str(tmp_path / "q4k_small.gguf"), 21, **SMALL)
    prompt = np.random.default_rng(3).integers(3, SMALL["vocab"], 16).tolist()
    res = _run(world, path, prompt, 16)
    ref = O.Model(path, threads=os.cpu_count() or 8)
    want_logits = ref.forward([prompt[0]], 0, ref.kv(8), algo=1)
    want_ids = ref.generate(prompt, len(prompt) + 16, fast=True).tolist()
    for r in range(world):
        assert _mar(res[r]["logits"], want_logits) <= 1e-4, r
        assert res[r]["ids"] == want_ids, r


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_70b_shape_two_layers_match_golden(world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import sys

    sys.path.insert(0, os.path.join(ROOT, "fishai-engine_b200"))
    import oracle as O
    from fishai_engine import synth

    g = json.load(open(os.path.join(ROOT, "tests", "golden", "70b2_greedy.json")))
    path = synth.cached_preset(g["preset"], **g["override"])
    prompt = g["prompt"]
    res = _run(world, path, prompt, len(g["greedy_ids"]), tc=True)
    ref = O.Model(path, threads=os.cpu_count() or 8)
    want, _ = ref.prefill(prompt, 0, ref.kv(len(prompt) + 8))
    for r in range(world):
        assert res[r]["ids"] == g["greedy_ids"], r
        assert _mar(res[r]["prefill_logits"], want) <= 1e-2, r
