"""Byte-level GGUF builders for tests (test infrastructure).

Restates the fixture builders of the reference's own unit tests so the same
files can be fed to the oracle and to the product parser:
  build_minimal_gguf      src/gguf.rs:809-847
  test_multi_tensor_gguf  src/gguf.rs:1273-1381
  build_test_gguf_file    src/model.rs:773-804
"""
import struct

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
MAGIC = 0x46465547


def gstr(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def kv_u32(key, v):
    return gstr(key) + struct.pack("<II", U32, v)


def kv_u64(key, v):
    return gstr(key) + struct.pack("<IQ", U64, v)


def kv_f32(key, v):
    return gstr(key) + struct.pack("<If", F32, v)


def kv_str(key, v):
    return gstr(key) + struct.pack("<I", STR) + gstr(v)


def tinfo(name, dims, ggml_type, offset):
    b = gstr(name) + struct.pack("<I", len(dims))
    for d in dims:
        b += struct.pack("<Q", d)
    return b + struct.pack("<IQ", ggml_type, offset)


def align(buf: bytes, a: int) -> bytes:
    pad = (-len(buf)) % a
    return buf + b"\x00" * pad


def header(n_tensors, n_kv, version=3, magic=MAGIC):
    return struct.pack("<IIQQ", magic, version, n_tensors, n_kv)


def minimal_gguf() -> bytes:
    b = header(1, 2) + kv_u32("general.alignment", 32) + kv_str("general.architecture", "testarch")
    b += tinfo("test.weight", [4, 8], 0, 0)
    b = align(b, 32)
    for i in range(32):
        b += struct.pack("<f", i * 0.5)
    return b


def multi_tensor_gguf() -> bytes:
    b = header(3, 6) + kv_u32("general.alignment", 64) + kv_str("general.architecture", "llama")
    b += kv_u64("llama.context_length", 4096) + kv_u64("llama.embedding_length", 4096)
    b += kv_u64("llama.block_count", 32) + kv_u64("llama.attention.head_count", 32)
    b += tinfo("token_embd.weight", [4096], 0, 0)
    b += tinfo("output_norm.weight", [4096], 0, 16384)
    b += tinfo("output.weight", [32000, 4096], 0, 32768)
    b = align(b, 64)
    b += b"".join(struct.pack("<f", float(i)) for i in range(4096))
    b += b"".join(struct.pack("<f", i * 2.0) for i in range(4096))
    return b


def model_config_gguf() -> bytes:
    b = header(0, 10) + kv_str("general.architecture", "llama")
    b += kv_u32("general.tokenizer.ggml.vocab_size", 32000) + kv_u32("llama.block_count", 32)
    b += kv_u32("llama.attention.head_count", 32) + kv_u32("llama.attention.head_count_kv", 32)
    b += kv_u32("llama.embedding_length", 4096) + kv_u32("llama.context_length", 2048)
    b += kv_f32("llama.attention.layer_norm_rms_epsilon", 1e-5) + kv_f32("llama.rope.freq_base", 10000.0)
    return align(b, 32)


def gqa_config_gguf() -> bytes:
    b = header(0, 7) + kv_str("general.architecture", "qwen2")
    b += kv_u32("general.tokenizer.ggml.vocab_size", 151936) + kv_u32("qwen2.block_count", 24)
    b += kv_u32("qwen2.attention.head_count", 28) + kv_u32("qwen2.attention.head_count_kv", 4)
    b += kv_u32("qwen2.embedding_length", 2048) + kv_u32("qwen2.context_length", 32768)
    return align(b, 32)


def tiny_llama_f32_gguf(n_embd=8, n_heads=2, n_kv=2, n_layers=1, vocab=16, n_ff=16, tied=True, scale=1.0):
    """create_test_model (src/model.rs:937-990) written as an F32 GGUF:
    arithmetic-ramp weights, norms 1.0, tied output."""
    tensors = []
    tensors.append(("token_embd.weight", [n_embd, vocab], [i * 0.01 * scale for i in range(vocab * n_embd)]))
    for l in range(n_layers):
        p = f"blk.{l}."
        qd, kvd = n_embd, n_kv * (n_embd // n_heads)
        tensors.append((p + "attn_norm.weight", [n_embd], [1.0] * n_embd))
        tensors.append((p + "attn_q.weight", [qd, n_embd], [i * 0.01 * scale for i in range(n_embd * qd)]))
        tensors.append((p + "attn_k.weight", [kvd, n_embd], [i * 0.02 * scale for i in range(n_embd * kvd)]))
        tensors.append((p + "attn_v.weight", [kvd, n_embd], [i * 0.03 * scale for i in range(n_embd * kvd)]))
        tensors.append((p + "attn_output.weight", [n_embd, qd], [i * 0.04 * scale for i in range(qd * n_embd)]))
        tensors.append((p + "ffn_norm.weight", [n_embd], [1.0] * n_embd))
        tensors.append((p + "ffn_gate.weight", [n_ff, n_embd], [i * 0.05 * scale for i in range(n_embd * n_ff)]))
        tensors.append((p + "ffn_up.weight", [n_ff, n_embd], [i * 0.06 * scale for i in range(n_embd * n_ff)]))
        tensors.append((p + "ffn_down.weight", [n_embd, n_ff], [i * 0.07 * scale for i in range(n_ff * n_embd)]))
    tensors.append(("output_norm.weight", [n_embd], [1.0] * n_embd))
    if not tied:
        tensors.append(("output.weight", [vocab, n_embd], [((i * 7) % 13 - 6) * 0.01 for i in range(vocab * n_embd)]))
    kvs = [kv_str("general.architecture", "llama"), kv_u32("general.tokenizer.ggml.vocab_size", vocab),
           kv_u32("llama.block_count", n_layers), kv_u32("llama.attention.head_count", n_heads),
           kv_u32("llama.attention.head_count_kv", n_kv), kv_u32("llama.embedding_length", n_embd),
           kv_u32("llama.context_length", 32), kv_f32("llama.feed_forward_length", float(n_ff)),
           kv_f32("llama.attention.layer_norm_rms_epsilon", 1e-5), kv_f32("llama.rope.freq_base", 10000.0)]
    b = header(len(tensors), len(kvs)) + b"".join(kvs)
    off = 0
    datas = []
    for name, dims, vals in tensors:
        b += tinfo(name, dims, 0, off)
        d = struct.pack(f"<{len(vals)}f", *vals)
        d = align(d, 32)
        datas.append(d)
        off += len(d)
    b = align(b, 32)
    return b + b"".join(datas)
