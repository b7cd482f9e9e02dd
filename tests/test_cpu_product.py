"""CPU-side tests of the product library (no GPU needed): the C ABI loads and
exports every declared entry point, the host GGUF reader and config logic
follow the reference's tests, the synthetic writer produces files the oracle
and gguf-py read, and GPU entry points fail loudly without a device."""
import json
import os
import re
import shutil

import numpy as np
import pytest

import gguf_bytes as gb
from fishai_engine import _lib as L
from fishai_engine import synth
from fishai_engine.gguf import GGUFFile
from fishai_engine.model import GenerationConfig, ModelConfig, ModelWeights
from fishai_engine.sampling import SamplerConfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _write(tmp_path, name, data):
    p = tmp_path / name
    p.write_bytes(data)
    return str(p)


def test_library_exports_every_declared_symbol():
    hdr = open(os.path.join(ROOT, "include", "fishai_cuda.h")).read()
    names = sorted(set(re.findall(r"^\s*(?:[a-z_ ]+\*?\s*\**)\b(fa_[a-z0-9_]+)\s*\(", hdr, re.M)))
    assert len(names) >= 40
    lib = L.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) <= set(L.SIGNATURES), sorted(set(names) - set(L.SIGNATURES))
    assert b"sm_100a" in lib.fa_version()


def test_python_constants_match_header():
    """Every #define FA_* of the C header has the same value in the ctypes
    mirror (status codes, ggml types, KV dtypes, debug keys)."""
    hdr = open(os.path.join(ROOT, "include", "fishai_cuda.h")).read()
    defs = {m.group(1): int(m.group(2)) for m in re.finditer(r"^#define FA_([A-Z0-9_]+) \(?(-?\d+)\)?", hdr, re.M)}
    assert len(defs) >= 20
    for name, val in defs.items():
        py = name[len("GGML_"):] if name.startswith("GGML_") else name
        assert hasattr(L, py), name
        assert getattr(L, py) == val, (name, getattr(L, py), val)


def test_gguf_minimal(tmp_path):  # src/gguf.rs:1041-1097
    g = GGUFFile.open(_write(tmp_path, "m.gguf", gb.minimal_gguf()))
    assert g.version == 3 and g.alignment == 32 and g.tensor_names() == ["test.weight"]
    assert g.model_architecture() == "testarch" and g.metadata_u64("general.alignment") == 32
    assert g.metadata_string("nonexistent.key") is None and g.metadata_f32("x") is None and g.metadata_bool("x") is None
    ti = g.tensor_info("test.weight")
    assert ti.dims == [4, 8] and ti.ggml_type == 0 and ti.nelement() == 32 and ti.shape() == [4, 8]
    raw = g.read_tensor_data(ti)
    assert np.frombuffer(raw, dtype=np.float32).tolist() == [i * 0.5 for i in range(32)]


def test_gguf_errors(tmp_path):  # src/gguf.rs:1100-1142, :1216-1227
    with pytest.raises(L.FishaiError, match="magic"):
        GGUFFile.open(_write(tmp_path, "a.gguf", gb.header(0, 0, magic=0xDEADBEEF)))
    with pytest.raises(L.FishaiError, match="version"):
        GGUFFile.open(_write(tmp_path, "b.gguf", gb.header(0, 0, version=99)))
    with pytest.raises(L.FishaiError, match="cannot open"):
        GGUFFile.open("/nonexistent/path/model.gguf")
    with pytest.raises(L.FishaiError):
        GGUFFile.open(_write(tmp_path, "c.gguf", gb.minimal_gguf()[:40]))  # truncated


def test_gguf_multi_tensor(tmp_path):  # src/gguf.rs:1272-1381
    g = GGUFFile.open(_write(tmp_path, "mt.gguf", gb.multi_tensor_gguf()))
    assert g.alignment == 64 and g.tensor_count() == 3
    assert (g.context_length(), g.embedding_length(), g.layer_count(), g.head_count()) == (4096, 4096, 32, 32)
    assert len(g.read_tensor_data("token_embd.weight")) == 16384
    assert len(g.read_tensor_data("output_norm.weight")) == 16384
    assert g.read_tensor_data("output.weight") == b""
    assert g.tensor_info("output.weight").nelement() == 32000 * 4096


def test_metadata_u64_from_u32(tmp_path):  # src/gguf.rs:1384-1421
    b = gb.align(gb.header(0, 2) + gb.kv_u32("general.alignment", 32) + gb.kv_u32("my_value", 100), 32)
    g = GGUFFile.open(_write(tmp_path, "u.gguf", b))
    assert g.metadata_u64("my_value") == 100 and g.metadata_i64("my_value") is None


def test_standard_magic_accepted(tmp_path):
    # files written by llama.cpp/gguf-py start with "GGUF" (0x46554747); the
    # reference's constant 0x46465547 reads "GUFF".  The product takes both.
    b = bytearray(gb.minimal_gguf())
    b[0:4] = b"GGUF"
    assert GGUFFile.open(_write(tmp_path, "s.gguf", bytes(b))).tensor_names() == ["test.weight"]


def test_model_config(tmp_path):  # src/model.rs:811-915, :1139-1153
    c = ModelConfig.from_gguf(GGUFFile.open(_write(tmp_path, "c.gguf", gb.model_config_gguf())))
    assert (c.n_layers, c.n_heads, c.n_kv_heads, c.n_embd, c.head_dim) == (32, 32, 32, 4096, 128)
    assert c.vocab_size == 32000 and c.context_len == 2048 and c.rope_freq_dim == 64
    assert abs(c.norm_eps - 1e-5) < 1e-8 and abs(c.rope_base - 10000.0) < 1e-3
    assert c.n_ff() == 11008  # default multiplier 2.667
    q = ModelConfig.from_gguf(GGUFFile.open(_write(tmp_path, "q.gguf", gb.gqa_config_gguf())))
    assert (q.n_heads, q.n_kv_heads, q.head_dim, q.n_layers) == (28, 4, 2048 // 28, 24)
    assert L.lib().fa_config_n_ff(256, 2.0) == 512 and L.lib().fa_config_n_ff(512, 2.0) == 1024
    assert L.lib().fa_config_n_ff(512, 1408 / 512) == 1536


def test_generation_and_sampler_defaults():  # src/model.rs:562-573, src/sampling.rs:31-80
    g = GenerationConfig()
    assert (g.max_tokens, g.temperature, g.top_k, g.top_p, g.repetition_penalty, g.stop_token_ids) == (
        512, 0.7, 40, 0.95, 1.15, [])
    assert SamplerConfig.greedy() == SamplerConfig(0.0, 0, 1.0, 1.0, 0.0, 0.0)
    assert SamplerConfig.precise().top_k == 20 and SamplerConfig.creative().temperature > 1.0


def test_synth_writer_readable_by_oracle_and_gguf_py(tmp_path, oracle):
    gguf = pytest.importorskip("gguf")
    from gguf.quants import dequantize as gdq

    p = synth.write(str(tmp_path / "kq.gguf"), 7, n_layers=1, n_embd=256, n_heads=4, n_kv_heads=4, n_ff=512,
                    vocab=512, context_len=64, rope_base=10000.0, norm_eps=1e-5, sigma=0.02,
                    type_embd=oracle.Q4_K, type_q=oracle.Q8_0, type_k=oracle.Q4_0, type_v=oracle.Q6_K,
                    type_o=oracle.F16, type_gate=oracle.Q4_K, type_up=oracle.Q4_K, type_down=oracle.Q6_K,
                    type_out=oracle.Q6_K)
    # the product reader and the oracle agree on the layout
    g, o = GGUFFile.open(p), oracle.GGUF(p)
    assert g.tensor_names() == o.tensor_names()
    for name in g.tensor_names():
        assert g.read_tensor_data(name) == o.read_tensor_data(name)
        ti = g.tensor_info(name)
        assert ti.dims == o.tensor_info(name)["dims"]
    cfg = ModelConfig.from_gguf(g)
    assert (cfg.n_embd, cfg.n_heads, cfg.vocab_size, cfg.n_ff()) == (256, 4, 512, 512)
    # gguf-py (standard magic) dequantises every tensor to the oracle's values
    std = str(tmp_path / "kq_std.gguf")
    shutil.copy(p, std)
    with open(std, "r+b") as f:
        f.write(b"GGUF")
    r = gguf.GGUFReader(std)
    for t in r.tensors:
        n = int(np.prod(t.shape))
        a = oracle.dequantize(o.read_tensor_data(t.name), int(t.tensor_type), n)
        b = gdq(np.array(t.data), t.tensor_type).reshape(-1).astype(np.float32)
        if int(t.tensor_type) == oracle.Q4_0:
            # ggml: element j = low nibble of byte j, j+16 = high nibble; the
            # reference: element 2j = high nibble, 2j+1 = low (src/quant.rs:143-148)
            g32 = b.reshape(-1, 32)
            b = np.stack([g32[:, 16:], g32[:, :16]], axis=2).reshape(-1)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), t.name
    # N(0, 0.02) weights
    w = oracle.dequantize(o.read_tensor_data("blk.0.ffn_gate.weight"), oracle.Q4_K, 256 * 512)
    assert 0.018 < float(w.std()) < 0.022


def test_synth_is_deterministic(tmp_path):
    a = synth.write_preset("tiny-q8_0", str(tmp_path / "a.gguf"), threads=2)
    b = synth.write_preset("tiny-q8_0", str(tmp_path / "b.gguf"), threads=5)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_tiny_golden_pins_oracle(oracle):
    gold = json.load(open(os.path.join(ROOT, "tests", "golden", "tiny_greedy.json")))
    path = synth.cached_preset(gold["preset"])
    m = oracle.Model(path, threads=os.cpu_count() or 4)
    assert m.cfg["n_ff_deviation"] == 1 and m.cfg["n_ff_used"] == 1408  # labelled deviation D2
    ids = m.generate(gold["prompt"], gold["prompt_len"] + len(gold["greedy_ids"]), fast=True).tolist()
    assert ids == gold["greedy_ids"]
    ids_ref = m.generate(gold["prompt"][:8], 8 + 4, fast=False).tolist()  # reference i-j-p order
    assert ids_ref == m.generate(gold["prompt"][:8], 8 + 4, fast=True).tolist()


def test_gpu_entry_points_fail_loudly_without_device(tmp_path):
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    p = synth.write_preset("tiny-q8_0", str(tmp_path / "t.gguf"))
    with pytest.raises(L.FishaiError) as e:
        ModelWeights.load_from_gguf(p)
    assert e.value.code == L.ERR_CUDA
