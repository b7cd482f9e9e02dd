"""Tensor-parallel sharding on the CPU, two gloo ranks (no GPU): each rank
takes its shards of one layer's weights through the library's own shard step
(fa_tp_shard, the code fa_model_load runs), dequantises them with the oracle
and runs its share of the layer (src/model.rs:347-423): column shards of
wq/wk/wv and gate/up, row shards of wo and down.  The all-reduce of the row
shards' partial sums (torch.distributed, gloo) must equal the unsharded
layer, and every shard must dequantise to exactly the matching slice of the
whole tensor.

Two weight sets: Q8_0 (32-column blocks) and Q4_K with 128-wide heads and two
KV heads, so each rank's K/V shard is half of a 256-column super-block (the
case eight-way parallelism meets on the 70B shape)."""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SPECS = {
    "q8_0": dict(n_layers=1, n_embd=512, n_heads=8, n_kv_heads=2, n_ff=1408, vocab=512, context_len=64,
                 rope_base=10000.0, norm_eps=1e-5, sigma=0.02, type_embd=8, type_q=8, type_k=8, type_v=8, type_o=8,
                 type_gate=8, type_up=8, type_down=8, type_out=8),
    "q4_k": dict(n_layers=1, n_embd=512, n_heads=4, n_kv_heads=2, n_ff=1024, vocab=512, context_len=64,
                 rope_base=500000.0, norm_eps=1e-5, sigma=0.015, type_embd=12, type_q=12, type_k=12, type_v=12,
                 type_o=12, type_gate=12, type_up=12, type_down=12, type_out=14),
}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(path):
    import oracle as O

    g = O.GGUF(path)
    out = {}
    for n in ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"):
        name = f"blk.0.{n}.weight"
        i = g.tensor_info(name)
        ne0, ne1 = i["dims"][:2]
        raw = np.frombuffer(g.read_tensor_data(name), dtype=np.uint8)
        out[n] = (i["ggml_type"], ne1, ne0, raw)  # type, K, N, native bytes
    return out


def _shard(L, t, raw, K, N, axis, rank, world):
    nb, rb = C.c_size_t(), C.c_uint32()
    L.check(L.lib().fa_tp_shard(t, raw.ctypes.data, K, N, axis, rank, world, None, 0, C.byref(nb), C.byref(rb)))
    out = np.zeros(nb.value, dtype=np.uint8)
    L.check(L.lib().fa_tp_shard(t, raw.ctypes.data, K, N, axis, rank, world, out.ctypes.data, out.size,
                                C.byref(nb), C.byref(rb)))
    return out, rb.value


def _deq(O, t, raw, K, N_stored, N_keep):
    return O.dequantize(raw.tobytes(), t, K * N_stored).reshape(K, N_stored)[:, :N_keep]


def _worker(rank, world, port, path, q):
    import sys

    for p in (os.path.join(ROOT, "fishai-engine_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    import torch

    import oracle as O
    from fishai_engine import _lib as L

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        W = _weights(path)
        full = {n: O.dequantize(r.tobytes(), t, K * N).reshape(K, N) for n, (t, K, N, r) in W.items()}
        rng = np.random.default_rng(1)
        d = W["attn_q"][1]
        xn = rng.normal(0, 1, d).astype(np.float32)
        errs = {}
        # column shards: each rank's slice of q / k / v / gate / up
        for n in ("attn_q", "attn_k", "attn_v", "ffn_gate", "ffn_up"):
            t, K, N, raw = W[n]
            sh, rb = _shard(L, t, raw, K, N, 1, rank, world)
            nc = N // world
            stored = rb // (34 if t == 8 else 144) * (32 if t == 8 else 256)
            w_loc = _deq(O, t, sh, K, stored, nc)
            errs[f"{n} slice"] = float(np.max(np.abs(w_loc - full[n][:, rank * nc:(rank + 1) * nc])))
        # row shards of wo / down, fed by this rank's columns of their inputs
        H = W["attn_q"][2]
        att = rng.normal(0, 1, H).astype(np.float32)
        g = (xn @ full["ffn_gate"]).astype(np.float32)
        u = (xn @ full["ffn_up"]).astype(np.float32)
        h = (g / (1.0 + np.exp(-g)) * u).astype(np.float32)
        for n, inp in (("attn_output", att), ("ffn_down", h)):
            t, K, N, raw = W[n]
            sh, rb = _shard(L, t, raw, K, N, 0, rank, world)
            nr = K // world
            w_loc = _deq(O, t, sh, nr, N, N)
            errs[f"{n} rows"] = float(np.max(np.abs(w_loc - full[n][rank * nr:(rank + 1) * nr])))
            part = torch.from_numpy((inp[rank * nr:(rank + 1) * nr].astype(np.float64) @ w_loc).astype(np.float32))
            dist.all_reduce(part)
            want = inp.astype(np.float64) @ full[n]
            errs[f"{n} all-reduce"] = float(np.max(np.abs(part.numpy() - want)) / np.max(np.abs(want)))
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("spec", list(SPECS))
def test_two_rank_shards_and_all_reduce_equal_the_unsharded_layer(spec, tmp_path):
    import sys

    sys.path.insert(0, os.path.join(ROOT, "fishai-engine_b200"))
    from fishai_engine import synth

    path = synth.write(str(tmp_path / f"{spec}.gguf"), 7, **SPECS[spec])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, errs in res.items():
        for k, v in errs.items():
            if "all-reduce" in k:
                assert v <= 1e-5, (rank, k, v)
            else:
                assert v == 0.0, (rank, k, v)  # shards dequantise bit for bit
