#!/usr/bin/env python
"""Decode throughput of the B200 token loop on the Llama-3-8B-shaped Q4_K_M
synthetic GGUF (32 layers, d 4096, 32/8 heads, FFN 14336, vocab 128256,
Q4_K with Q6_K attn_v / ffn_down / output, weights N(0, 0.02) from seed 2):
batch 1, a 2048-token prompt, then greedy decode.  One step = one decode
token (one forward pass through the model + argmax, a CUDA-graph replay).

Generation follows GenerationState::generate (src/model.rs:638-705): the
prompt is prefilled, the last prompt token is fed again at position P, and
the greedy ids that follow are checked against the committed 64-id golden
before the timed steps continue the same sequence.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --profile gateup --layers 2 --reps 3   # one GEMV kind on a
      reduced-depth model of the same shapes (small cases for ncu captures)

With N > 1 (torchrun) every rank runs an independent replica of the 8B b=1
decode (it does not shard); value = all ranks' tokens / max rank time.  The
"tp70b" key carries the 70B-shaped model tensor-parallel over the same N
GPUs (NCCL all-reduce after every o and down projection); at N = 1 it is
that model on one GPU.  Prints one JSON line (rank 0)."""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "fishai-engine_b200"))

METRIC = "decode tok/s at 8B Q4_K_M (b=1)"
PRESET = "llama3-8b-q4_k_m"
BATCH_PRESET = "llama3-8b-q8_0"
BATCH_WORKLOAD = "llama3-8b-shaped Q8_0 synthetic GGUF (seed 3), 64 sequences x 4096-token prompts, 128 sampled steps"
WORKLOAD = "llama3-8b-shaped Q4_K_M synthetic GGUF, batch 1, 2048-token prompt, greedy decode"
DATA = "synthetic (seeded N(0,0.02) weights, uniform prompt ids)"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")
# the other workload shapes, each reported at one GPU beside the headline:
# name -> (preset, override, prompt seed, prompt, greedy tokens, golden file)
EXTRA = {
    "tiny": ("tiny-q8_0", {}, 0, 32, 128, "tiny_greedy.json"),
    "7b": ("llama2-7b-q4_0", {}, 1, 512, 256, "7b_greedy.json"),
    "70b": ("llama3-70b-q4_k", {}, 4, 4096, 256, None),
}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d.get("hbm_gbs", FALLBACK_HBM_GBS)), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak():
    """dense 16-bit tensor peak (TFLOP/s): the measured burst figure for kernels timed alone"""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured"
    return FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def load_golden(name):
    p = os.path.join(GOLDEN_DIR, name) if name else None
    if not p or not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f)


def golden_check(golden, prompt, ids):
    """{match, checked, first_mismatch} of generated ids against a committed
    golden (None when the golden does not cover this prompt)"""
    if not golden or golden["prompt"] != list(prompt):
        return None
    want = golden["greedy_ids"]
    n = min(len(want), len(ids))
    bad = [i for i in range(n) if int(ids[i]) != int(want[i])]
    return {"match": not bad and n == len(want), "checked": n, "first_mismatch": bad[0] if bad else None}


def cpu_token_sample(path, prompt_len, layers, threads):
    """Reference-order CPU timing (the oracle port; one thread, as the
    reference runs): one decode token at context prompt_len through the first
    `layers` layers (all when 0) -- matmuls in i-j-p order, RoPE, the K/V head
    expansion copy, attention over the whole cache -- plus the output head and
    the greedy pick.  Returns (seconds per whole token, layer seconds, head
    seconds, layers timed, model layers)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    m = O.Model(path, resident=False, threads=threads)
    L = m.cfg["n_layers"]
    n = layers if 0 < layers < L else L
    kv = m.kv(prompt_len + 2)
    kv.fill_synthetic(prompt_len)
    ls, hs, _ = m.time_token(kv, 5, prompt_len, n)
    del kv
    m.close()
    return hs + ls * L / n, ls, hs, n, L


def reference_arm(args, world, rank):
    """The reference's own CPU algorithm for the headline workload, timed on
    this host: the oracle (the reference crate cannot be built: no Rust
    toolchain) runs whole decode tokens of the 8B Q4_K_M model at context
    2048 in the reference's loop order on one thread.  The input file is
    written by the oracle's copy of the synthetic writer, so this arm never
    loads the CUDA library."""
    if rank != 0:
        return 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O

    from fishai_engine import synth

    path = synth.cached_preset(PRESET, writer=O.write_gguf)
    m = O.Model(path, resident=False, threads=os.cpu_count() or 1)
    P, n_tok = args.prompt, max(1, args.ref_tokens)
    kv = m.kv(P + n_tok + 2)
    kv.fill_synthetic(P)
    tok = int(np.random.default_rng(2).integers(3, m.cfg["vocab_size"], P)[-1])
    t_layers = t_head = 0.0
    for i in range(n_tok):
        ls, hs, tok = m.time_token(kv, tok, P + i, 0)
        t_layers += ls
        t_head += hs
    total = t_layers + t_head
    value = n_tok / total
    sample = (f"{n_tok} whole decode token(s) at context {P}: all {m.cfg['n_layers']} layers (i-j-p f32 matmuls, "
              f"RoPE, expand_kv_heads copy, attention) {t_layers:.1f}s + output head and greedy pick {t_head:.1f}s, "
              f"one thread (host has {os.cpu_count()} cores); weights dequantised to f32 outside the timed region, "
              f"as the reference does at load; cache rows before position {P} hold synthetic values")
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": n_tok,
            "steps_requested": args.steps, "warmup": 0, "ms_per_step": 1000.0 * total / n_tok,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": DATA,
            "config": {"workload": WORKLOAD, "batch": 1, "prompt": P}, "impl": "reference",
            "timed": "every step is one whole decode token; nothing is extrapolated",
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": 1, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    m.close()
    print(json.dumps(line), flush=True)
    return 0


PROFILE_KINDS = {"qkv": 0, "o": 1, "gateup": 2, "down": 3, "head": 4}


def profile_one(args):
    """Launch one GEMV kind `reps` times over every layer of a reduced-depth
    model with the benchmark's shapes and types; print its device time."""
    import ctypes as C

    from fishai_engine import synth, _lib as L
    from fishai_engine.model import ModelWeights

    path = synth.cached_preset(PRESET, n_layers=args.layers)
    m = ModelWeights.load_from_gguf(path)
    avg, nbytes = C.c_float(), C.c_uint64()
    L.check(L.lib().fa_profile_gemv(m._h, PROFILE_KINDS[args.profile], args.reps, C.byref(avg), C.byref(nbytes)))
    print(json.dumps({"profile": args.profile, "layers": args.layers, "reps": args.reps,
                      "avg_launch_us": avg.value * 1000.0, "bytes_per_launch": nbytes.value,
                      "achieved_gbs": nbytes.value / (avg.value / 1000.0) / 1e9}), flush=True)
    m.close()
    return 0


def profile_gemm(args):
    """One tcgen05 token GEMM (the prefill / batched-decode projection) of a
    reduced-depth model with the benchmark's shapes: device time and TFLOP/s."""
    import ctypes as C

    from fishai_engine import synth, _lib as L
    from fishai_engine.model import ModelWeights

    path = synth.cached_preset(BATCH_PRESET if args.batch_weights else PRESET, n_layers=args.layers)
    m = ModelWeights.load_from_gguf(path)
    ms, fl = C.c_float(), C.c_double()
    L.check(L.lib().fa_profile_gemm(m._h, PROFILE_KINDS[args.profile_gemm], 0, args.tokens, args.reps, C.byref(ms),
                                    C.byref(fl)))
    print(json.dumps({"profile_gemm": args.profile_gemm, "weights": BATCH_PRESET if args.batch_weights else PRESET,
                      "tokens": args.tokens, "layers": args.layers,
                      "reps": args.reps, "avg_launch_us": ms.value * 1000.0, "flops": fl.value,
                      "tflops": fl.value / (ms.value / 1000.0) / 1e12}), flush=True)
    m.close()
    return 0


def profile_kernels(args):
    """A compact workload that launches every token-path kernel class a few
    times, for ncu captures (one kernel per capture with -k): a 2048-token
    tensor-core prefill of a one-layer 8B-shaped Q4_K_M model (RMSNorm rows,
    token GEMMs with their split fixups, RoPE + KV append, causal flash
    attention, SwiGLU rows), then two batched decode steps of 64 sequences at
    context 256 on the one-layer Q8_0 model (batched RoPE, decode attention,
    the sampler with T 0.8 / top-k 40 / top-p 0.9)."""
    import numpy as np

    from fishai_engine import synth, _lib as L
    from fishai_engine.model import ModelWeights
    from fishai_engine.sampling import Sampler, SamplerConfig

    m = ModelWeights.load_from_gguf(synth.cached_preset(PRESET, n_layers=1), use_tc_prefill=True)
    V = m.config.vocab_size
    prompt = np.random.default_rng(2).integers(3, V, 2048).tolist()
    m.prefill(prompt, 0, m.new_kv_cache(2056, dtype=L.KV_F16), want_logits=False)
    m.close()
    mb = ModelWeights.load_from_gguf(synth.cached_preset(BATCH_PRESET, n_layers=1), use_tc_prefill=True)
    B, P = 64, 256
    kv = mb.new_kv_cache(P + 16, dtype=L.KV_F16, n_seq=B)
    rng = np.random.default_rng(3)
    last = []
    for r in range(B):
        pr = rng.integers(3, V, P).tolist()
        mb.prefill(pr, 0, kv, seq=r, want_logits=False)
        last.append(pr[-1])
    smp = Sampler(SamplerConfig(0.8, 40, 0.9, 1.0, 0.0, 0.0), V, seeds=[1000 + r for r in range(B)])
    ids = mb.decode_batch(kv, last, [P] * B, smp, 2)
    mb.close()
    print(json.dumps({"profile_kernels": "ok", "ids": ids[-1][:4].tolist()}), flush=True)
    return 0


def kv_read_bytes(cfg, kv_elem, ctx):
    return 2 * cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * kv_elem * ctx


def greedy_config(name, args, local, peak):
    """One more workload shape at one GPU: prefill, re-feed of the last
    prompt token at position P, then G greedy steps timed with CUDA events;
    the ids are checked against the shape's golden where one is committed."""
    import numpy as np
    import torch

    from fishai_engine import synth, _lib as L
    from fishai_engine.model import ModelWeights

    preset, override, seed, P, G, gname = EXTRA[name]
    path = synth.cached_preset(preset, **override)
    m = ModelWeights.load_from_gguf(path, device=local, use_tc_prefill=args.decode_prefill == "tc")
    cfg = m.config
    _, wbytes = m.weight_bytes()
    prompt = np.random.default_rng(seed).integers(3, cfg.vocab_size, P).tolist()
    kv_dtype = L.KV_F16 if args.kv == "f16" else L.KV_F32
    kv = m.new_kv_cache(P + G + 8, dtype=kv_dtype)
    stream = torch.cuda.ExternalStream(L.lib().fa_model_stream(m._h))
    t0 = time.perf_counter()
    m.prefill(prompt, 0, kv, want_logits=False)
    prefill_s = time.perf_counter() - t0
    m.decode_greedy(m.new_kv_cache(8, dtype=kv_dtype), prompt[-1], 0, 4)  # graph capture outside the timing
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    ids = m.decode_greedy(kv, prompt[-1], P, G)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    mean_ctx = P + (G + 1) / 2.0
    step_bytes = wbytes + kv_read_bytes(cfg, 2 if args.kv == "f16" else 4, mean_ctx)
    gbs = step_bytes * G / (ms / 1000.0) / 1e9
    out = {"value": G / (ms / 1000.0), "unit": "tok/s", "model": f"{preset} synthetic GGUF (seed {seed})",
           "batch": 1, "prompt": P, "steps": G, "ms_per_step": ms / G, "kv_cache": args.kv,
           "prefill": args.decode_prefill, "prefill_wall_s": prefill_s,
           "greedy_ids_match_golden": golden_check(load_golden(gname), prompt, ids),
           "roofline": {"bound": "hbm", "bytes_per_step": step_bytes, "achieved_gbs": gbs, "peak": peak,
                        "unit": "GB/s", "frac": gbs / peak}}
    del kv
    m.close()
    return out


TP_PRESET = "llama3-70b-q4_k"


def tp70b_leg(args, world, rank, local, pg, peak):
    """Config 5: the Llama-3-70B-shaped Q4_K model (Q6_K head, seed 4) on
    all ranks of the job as one tensor-parallel model (TP = world; world 1 is
    the single-GPU figure): a 4096-token prompt through the tensor-core
    prefill, the last prompt token fed again, greedy decode timed with CUDA
    events (max over ranks); then 16 sequences of 2048-token contexts decoding
    together.  Every rank computes the same ids (replicated head)."""
    import numpy as np
    import torch

    from fishai_engine import synth, _lib as L
    from fishai_engine.model import ModelWeights, tp_unique_id
    from fishai_engine.sampling import Sampler, SamplerConfig

    over = {"n_layers": args.tp_layers} if args.tp_layers else {}
    if rank == 0:
        synth.cached_preset(TP_PRESET, **over)
    if pg:
        pg.barrier()
    path = synth.cached_preset(TP_PRESET, **over)
    uid = None
    if world > 1:
        box = [tp_unique_id() if rank == 0 else None]
        pg.broadcast_object_list(box, src=0)
        uid = box[0]
    t0 = time.perf_counter()
    m = ModelWeights.load_from_gguf(path, device=local, tp_rank=rank, tp_world=world, nccl_id=uid,
                                    use_tc_prefill=True)
    load_s = time.perf_counter() - t0
    cfg = m.config
    _, wbytes = m.weight_bytes()
    P, G, K = 4096, 8, args.tp_steps
    prompt = np.random.default_rng(4).integers(3, cfg.vocab_size, P).tolist()
    kv = m.new_kv_cache(P + G + K + 8, dtype=L.KV_F16)
    stream = torch.cuda.ExternalStream(L.lib().fa_model_stream(m._h))
    t0 = time.perf_counter()
    m.prefill(prompt, 0, kv, want_logits=False)
    prefill_s = time.perf_counter() - t0
    ids = m.decode_greedy(kv, prompt[-1], P, G)  # warm-up: graph capture, NCCL connections
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    ids2 = m.decode_greedy(kv, int(ids[-1]), P + G, K)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    agree = True
    if pg:
        t = torch.tensor([ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
        mine = torch.tensor(ids2.astype(np.int64), device="cuda")
        first = mine.clone()
        pg.broadcast(first, src=0)
        ok = torch.tensor([int(torch.equal(mine, first))], device="cuda")
        pg.all_reduce(ok, op=pg.ReduceOp.MIN)
        agree = bool(ok.item())
    mean_ctx = P + G + (K + 1) / 2.0
    hd = cfg.head_dim
    kv_local = 2 * cfg.n_layers * m.local_kv_heads * hd * 2 * mean_ctx
    gpu_bytes = wbytes + kv_local  # what one GPU streams per token (its shards + replicated head)
    gbs = gpu_bytes * K / (ms / 1000.0) / 1e9
    out = {"value": K / (ms / 1000.0), "unit": "tok/s",
           "model": f"{TP_PRESET} synthetic GGUF (seed 4)" + (f", first {args.tp_layers} layers" if over else ""),
           "tp": world, "batch": 1, "prompt": P, "steps": K, "ms_per_step": ms / K, "kv_cache": "f16",
           "prefill": "tc", "prefill_wall_s": prefill_s, "load_s": load_s, "ranks_agree_on_ids": agree,
           "all_reduces_per_token": 2 * cfg.n_layers if world > 1 else 0,
           "roofline": {"bound": "hbm", "bytes_per_gpu_per_step": gpu_bytes, "achieved_gbs_per_gpu": gbs,
                        "peak": peak, "unit": "GB/s", "frac": gbs / peak}}
    del kv
    # 16 sequences with 2048-token contexts, greedy, decoding together
    B, Pb, Kb = 16, 2048, args.tp_batch_steps
    if Kb > 0:
        kvb = m.new_kv_cache(Pb + Kb + 16, dtype=L.KV_F16, n_seq=B)
        rng = np.random.default_rng(4)
        last = []
        for r in range(B):
            pr = rng.integers(3, cfg.vocab_size, Pb).tolist()
            m.prefill(pr, 0, kvb, seq=r, want_logits=False)
            last.append(pr[-1])
        smp = Sampler(SamplerConfig(0.0, 0, 1.0, 1.0, 0.0, 0.0), cfg.vocab_size, seeds=list(range(B)))
        w = m.decode_batch(kvb, last, [Pb] * B, smp, 2)
        if pg:
            pg.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        m.decode_batch(kvb, w[-1].tolist(), [Pb + 2] * B, smp, Kb)
        e1.record(stream)
        e1.synchronize()
        bms = e0.elapsed_time(e1)
        if pg:
            t = torch.tensor([bms], device="cuda")
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            bms = float(t.item())
        bkv = 2 * cfg.n_layers * m.local_kv_heads * hd * 2 * (Pb + 2 + (Kb + 1) / 2.0) * B
        bgbs = (wbytes + bkv) * Kb / (bms / 1000.0) / 1e9
        out["b16"] = {"value": B * Kb / (bms / 1000.0), "unit": "tok/s", "batch": B, "context": Pb, "steps": Kb,
                      "ms_per_step": bms / Kb, "sampler": "greedy",
                      "roofline": {"bound": "hbm", "bytes_per_gpu_per_step": wbytes + bkv,
                                   "achieved_gbs_per_gpu": bgbs, "peak": peak, "unit": "GB/s", "frac": bgbs / peak}}
        del kvb, smp
    m.close()
    if rank == 0 and world == 1 and args.cpu_layers > 0:
        per_tok, ls, hs, n, nl = cpu_token_sample(path, P, 1, os.cpu_count() or 1)
        out["cpu_baseline"] = {"value": 1.0 / per_tok, "unit": "tok/s", "cores": 1, "kind": "port",
                               "sample": f"one decode token at context {P} in the reference's order on one core: "
                                         f"1 of {nl} layers {ls:.1f}s + output head and greedy pick {hs:.1f}s; "
                                         f"per-token time = head + layer x {nl}"}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--kv", choices=["f16", "f32"], default="f16")
    ap.add_argument("--decode-prefill", choices=["tc", "exact"], default="exact",
                    help="how the prompt of the timed decode is prefilled: exact (f32 token steps, the reference's "
                         "values) or tc (f16 tensor cores)")
    ap.add_argument("--cpu-layers", type=int, default=8,
                    help="layers of the whole-token CPU sample beside our figure (0: skip)")
    ap.add_argument("--ref-tokens", type=int, default=1, help="whole decode tokens the reference arm times")
    ap.add_argument("--configs", default="tiny,7b",
                    help="other workload shapes reported at one GPU (tiny, 7b; empty: none)")
    ap.add_argument("--tp70b", type=int, choices=[0, 1], default=1,
                    help="1: the 70B-shaped model, tensor-parallel over all ranks of the job (one GPU at N=1)")
    ap.add_argument("--tp-steps", type=int, default=128, help="timed greedy steps of the 70B leg")
    ap.add_argument("--tp-batch-steps", type=int, default=32, help="timed steps of the 70B b=16 leg (0: skip)")
    ap.add_argument("--tp-layers", type=int, default=0,
                    help="reduced-depth 70B-shaped model for quick checks (0: all 80 layers)")
    ap.add_argument("--batch", type=int, default=64, help="sequences of the batched-decode figure (0: skip)")
    ap.add_argument("--batch-prompt", type=int, default=4096)
    ap.add_argument("--batch-steps", type=int, default=128)
    ap.add_argument("--step-kernel", type=int, choices=[0, 1], default=0,
                    help="1: each decode step is one persistent kernel launch")
    ap.add_argument("--profile", choices=list(PROFILE_KINDS), default=None,
                    help="time one GEMV kind only, on a model with --layers layers")
    ap.add_argument("--profile-gemm", choices=list(PROFILE_KINDS), default=None,
                    help="time one tcgen05 token GEMM of a reduced-depth model (--layers) for --tokens tokens")
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--batch-weights", action="store_true",
                    help="--profile-gemm on the Q8_0 model of the batched-decode workload")
    ap.add_argument("--model-layers", type=int, default=0,
                    help="reduced-depth model of the same shapes for the whole run (0: the full 32 layers)")
    ap.add_argument("--profile-kernels", action="store_true",
                    help="a compact workload launching every token-path kernel class (for ncu captures)")
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    if args.profile:
        return profile_one(args)
    if args.profile_gemm:
        return profile_gemm(args)
    if args.profile_kernels:
        return profile_kernels(args)
    world, rank, local = dist_env()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return reference_arm(args, world, rank)

    import ctypes as C

    import numpy as np
    import torch

    from fishai_engine import synth, _lib as L
    from fishai_engine.model import ModelWeights

    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(minutes=10))
        pg = dist
    # the synthetic model: rank 0 writes it once, others wait
    ml = {"n_layers": args.model_layers} if args.model_layers else {}
    if rank == 0:
        path = synth.cached_preset(PRESET, **ml)
    if pg:
        pg.barrier()
    path = synth.cached_preset(PRESET, **ml)

    m = ModelWeights.load_from_gguf(path, device=local, use_step_kernel=bool(args.step_kernel),
                                    use_tc_prefill=True)
    cfg = m.config
    step_kernel = m.step_kernel_active
    dev_bytes, step_weight_bytes = m.weight_bytes()
    P, K, W = args.prompt, args.steps, args.warmup
    G = 64  # greedy ids checked against the golden before the warm-up
    E = min(K, 128)  # end-to-end steps
    kv_dtype = L.KV_F16 if args.kv == "f16" else L.KV_F32
    prompt = np.random.default_rng(2 + rank).integers(3, cfg.vocab_size, P).tolist()
    stream = torch.cuda.ExternalStream(L.lib().fa_model_stream(m._h))
    peak, peak_src = measured_peaks()

    # prefill throughput on the tensor-core path (scratch caches: one warm-up
    # run for the workspace and tensor maps, then the timed run)
    kv_w = m.new_kv_cache(P + 8, dtype=kv_dtype)
    m.prefill(prompt, 0, kv_w, want_logits=False)
    del kv_w
    kv_p = m.new_kv_cache(P + 8, dtype=kv_dtype)
    torch.cuda.synchronize()
    pe0, pe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pe0.record(stream)
    t0 = time.perf_counter()
    m.prefill(prompt, 0, kv_p)
    prefill_s = time.perf_counter() - t0
    pe1.record(stream)
    pe1.synchronize()
    prefill_dev_s = pe0.elapsed_time(pe1) / 1000.0
    del kv_p

    # the decode sequence: prompt prefilled (--decode-prefill), the last
    # prompt token fed again at position P (src/model.rs:656-657), greedy ids
    # checked against the golden, then warm-up and timed steps continue it
    m.set_tc_prefill(args.decode_prefill == "tc")
    kv = m.new_kv_cache(P + G + W + K + E + 8, dtype=kv_dtype)
    t0 = time.perf_counter()
    m.prefill(prompt, 0, kv, want_logits=False)
    decode_prefill_s = time.perf_counter() - t0
    ids = m.decode_greedy(kv, prompt[-1], P, G)
    parity = golden_check(load_golden("8b_greedy.json") if not ml else None, prompt, ids)
    pos = P + G
    ids = m.decode_greedy(kv, int(ids[-1]), pos, W)  # warm-up (steady state)
    pos += W
    tok = int(ids[-1])

    clock = ClockSampler(local)
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    clock.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    ids = m.decode_greedy(kv, tok, pos, K)
    ev1.record(stream)
    ev1.synchronize()
    torch.cuda.synchronize()
    clocks = clock.stop()
    if pg:
        pg.barrier()
    ms = ev0.elapsed_time(ev1)
    launches = m.step_launches()
    pos += K
    tok = int(ids[-1])
    t_max = ms
    if pg:
        t = torch.tensor([ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        t_max = float(t.item())
    value = world * K / (t_max / 1000.0)

    # end to end through the public API: per step one token id in and the
    # argmax id out (fa_forward with no logits buffer; the library moves the
    # 40-byte step state each way through a pinned staging buffer)
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    t0 = time.perf_counter()
    for _ in range(E):
        _, am = m.forward([tok], pos, kv, return_argmax=True, want_logits=False)
        tok = int(am[0])
        pos += 1
    e2e_s = time.perf_counter() - t0
    e2e_local = torch.tensor([e2e_s], device="cuda")
    if pg:
        pg.all_reduce(e2e_local, op=pg.ReduceOp.MAX)
    e2e_value = world * E / float(e2e_local.item())

    # roofline of the dominant kernel: the fused FFN gate+up GEMV
    # (33% of a step's bytes), timed with CUDA events over all 32 layers
    avg, nbytes = C.c_float(), C.c_uint64()
    L.check(L.lib().fa_profile_gemv(m._h, 2, 64, C.byref(avg), C.byref(nbytes)))
    achieved = nbytes.value / (avg.value / 1000.0) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "gemv_gateup_8b_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get("bytes_per_launch")
    head_avg, head_bytes = C.c_float(), C.c_uint64()
    L.check(L.lib().fa_profile_gemv(m._h, 4, 8, C.byref(head_avg), C.byref(head_bytes)))

    # whole-step bytes: weights + embedding row + KV read at the mean context
    kv_elem = 2 if args.kv == "f16" else 4
    ctx0 = P + G + W
    mean_ctx = ctx0 + (K + 1) / 2.0
    step_bytes = step_weight_bytes + kv_read_bytes(cfg, kv_elem, mean_ctx)
    step_gbs = step_bytes * (K / (ms / 1000.0)) / 1e9

    # prefill roofline: tensor-bound; linear flops 2 x (layer weights) per token
    # plus causal attention 4 L Hq hd P(P+1)/2, against the measured dense peak
    d, hd, F = cfg.n_embd, cfg.head_dim, cfg.n_ff_used
    lin = cfg.n_layers * (d * cfg.n_heads * hd * 2 + 2 * d * cfg.n_kv_heads * hd + 3 * d * F)
    pf_flops = 2.0 * lin * P + 4.0 * cfg.n_layers * cfg.n_heads * hd * P * (P + 1) / 2 + 2.0 * d * cfg.vocab_size
    tpeak, tpeak_src = measured_tensor_peak()
    gemm_ms, gemm_fl = C.c_float(), C.c_double()
    L.check(L.lib().fa_profile_gemm(m._h, 2, 0, P, 5, C.byref(gemm_ms), C.byref(gemm_fl)))
    gemm = {"kernel": "k_qgemm (gate+up, Q4_K, tcgen05 f16)", "tokens": P, "avg_launch_us": gemm_ms.value * 1e3,
            "achieved": gemm_fl.value / (gemm_ms.value / 1000.0) / 1e12, "peak": tpeak, "unit": "TFLOP/s",
            "frac": gemm_fl.value / (gemm_ms.value / 1000.0) / 1e12 / tpeak}
    prefill = {"value": P / prefill_s, "unit": "tok/s", "tokens": P,
               "path": "f16 tensor cores: tcgen05 dequant-GEMMs, causal flash attention (mma.sync), chunks of 2048",
               "device_s": prefill_dev_s,
               "roofline": {"bound": "tensor", "flops": pf_flops, "achieved": pf_flops / prefill_dev_s / 1e12,
                            "peak": tpeak, "unit": "TFLOP/s", "frac": pf_flops / prefill_dev_s / 1e12 / tpeak,
                            "peak_source": tpeak_src},
               "gemm": gemm}
    m.close()

    tp70b = tp70b_leg(args, world, rank, local, pg, peak) if args.tp70b and not ml else None

    # batched decode on the 8B Q8_0 model (seed 3): 64 sequences with
    # 4096-token prompts prefilled into the paged f16 cache, then 128 steps
    # sampled with T 0.8, top-k 40, top-p 0.9 (Philox seed 1000 + i), all
    # sequences one token per step
    batch = None
    if args.batch > 0 and world == 1:
        from fishai_engine.sampling import Sampler, SamplerConfig

        if rank == 0:
            synth.cached_preset(BATCH_PRESET, **ml)
        if pg:
            pg.barrier()
        mb = ModelWeights.load_from_gguf(synth.cached_preset(BATCH_PRESET, **ml), device=local, use_tc_prefill=True)
        _, b_weight_bytes = mb.weight_bytes()
        bstream = torch.cuda.ExternalStream(L.lib().fa_model_stream(mb._h))
        B, Pb, Kb = args.batch, args.batch_prompt, args.batch_steps
        kvb = mb.new_kv_cache(Pb + Kb + 16, dtype=L.KV_F16, n_seq=B)
        rngb = np.random.default_rng(3)
        first = []
        t0 = time.perf_counter()
        for r in range(B):
            pr = rngb.integers(3, cfg.vocab_size, Pb).tolist()
            mb.prefill(pr, 0, kvb, seq=r, want_logits=False)
            first.append(pr[-1])
        pf_b = time.perf_counter() - t0
        smp = Sampler(SamplerConfig(0.8, 40, 0.9, 1.0, 0.0, 0.0), cfg.vocab_size, seeds=[1000 + r for r in range(B)])
        warm = 4
        ids_w = mb.decode_batch(kvb, first, [Pb] * B, smp, warm)
        toks, poss = ids_w[-1].tolist(), [Pb + warm] * B
        torch.cuda.synchronize()
        be0, be1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        be0.record(bstream)
        mb.decode_batch(kvb, toks, poss, smp, Kb)
        be1.record(bstream)
        be1.synchronize()
        b_ms = be0.elapsed_time(be1)
        mean_ctx_b = Pb + warm + (Kb + 1) / 2.0
        kvb_bytes = kv_read_bytes(cfg, 2, mean_ctx_b) * B
        b_step_bytes = b_weight_bytes + kvb_bytes
        b_gbs = b_step_bytes * Kb / (b_ms / 1000.0) / 1e9
        batch = {"value": B * Kb / (b_ms / 1000.0), "unit": "tok/s", "model": BATCH_WORKLOAD, "batch": B,
                 "prompt": Pb, "steps": Kb,
                 "warmup": warm, "ms_per_step": b_ms / Kb, "kv_cache": "f16",
                 "sampler": "T 0.8, top-k 40, top-p 0.9, Philox4x32-10 seed 1000+i per sequence",
                 "path": "f16 tcgen05 GEMMs at T=64 (split K), mma.sync split-K decode attention per row, device sampler",
                 "prefill_s": pf_b,
                 "roofline": {"bound": "hbm", "bytes_per_step": b_step_bytes, "achieved_gbs": b_gbs, "peak": peak,
                              "unit": "GB/s", "frac": b_gbs / peak}}
        del kvb, smp
        mb.close()

    extra = {}
    if not ml and world == 1:
        for name in [c for c in args.configs.split(",") if c]:
            extra[name] = greedy_config(name, args, local, peak)

    cpu = None
    if rank == 0 and world == 1 and args.cpu_layers > 0:
        per_tok, ls, hs, n, nl = cpu_token_sample(path, P, args.cpu_layers, os.cpu_count() or 1)
        cpu = {"value": 1.0 / per_tok, "unit": "tok/s", "cores": 1, "kind": "port",
               "sample": f"one decode token at context {P} in the reference's order on one core: {n} of {nl} layers "
                         f"(i-j-p f32 matmuls, RoPE, expand_kv_heads copy, attention) {ls:.1f}s + output head and "
                         f"greedy pick {hs:.1f}s; per-token time = head + layers x {nl}/{n}; host has "
                         f"{os.cpu_count()} cores"}

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": t_max / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 activations, Q4_K/Q6_K weights, f16 KV" if args.kv == "f16" else "f32",
        "data": DATA,
        "config": {"workload": WORKLOAD, "batch": 1, "prompt": P, "kv_cache": args.kv,
                   "decode_prefill": args.decode_prefill, "step_kernel": step_kernel,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (4.9 GB of weights streamed per step)"},
        "greedy_ids_match_golden": parity,
        "roofline": {"bound": "hbm", "kernel": "k_gemv_mma (fused ffn gate+up, Q4_K)", "achieved": achieved,
                     "peak": peak, "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                     "bytes_per_launch": nbytes.value, "avg_launch_us": avg.value * 1000.0,
                     "peak_source": peak_src,
                     "step": {"bytes_per_step": step_bytes, "achieved_gbs": step_gbs, "frac": step_gbs / peak},
                     "head": {"bytes_per_launch": head_bytes.value, "avg_launch_us": head_avg.value * 1000.0,
                              "achieved_gbs": head_bytes.value / (head_avg.value / 1000.0) / 1e9}},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 40, "d2h_bytes_per_step": 40,
                "api": "fa_forward with no logits buffer: the step state (token id, position) in and the argmax "
                       "id out, 40 bytes each way through the library's pinned staging buffer"},
        "prefill": prefill,
        "decode_b64": batch,
        "configs": extra,
        "tp70b": tp70b,
        "gpu_launches": launches * K,
        "launches_per_step": launches,
        "clocks": clocks,
        "decode_prefill_wall_s": decode_prefill_s,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del kv
    if pg:
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
