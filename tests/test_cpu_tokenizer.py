"""BpeTokenizer (src/tokenizer.rs) through the C ABI, on the host: the
reference's own unit tests (src/tokenizer.rs:620-1100) on the same fixture
vocabulary, plus the GGUF wiring (tokenizer.ggml.* arrays and config keys)
and the pre-tokenizer's leftmost-first rules."""
import struct

import pytest

from fishai_engine.tokenizer import BYTE, CONTROL, NORMAL, BpeTokenizer, TokenizerConfig
from gguf_bytes import ARR, BOOL, F32, I32, STR, U32, gstr, header

NORMAL_CHARS = " abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ.,!?"


def fixture_vocab():
    """make_test_tokenizer (src/tokenizer.rs:620-828): <unk> <s> </s>, 256
    byte tokens, the normal characters, then ab abc he llo ll lo"""
    toks, types, scores = ["<unk>", "<s>", "</s>"], [CONTROL] * 3, [0.0] * 3
    for b in range(256):
        toks.append(f"<0x{b:02X}>")
        types.append(BYTE)
        scores.append(0.0)
    for ch in NORMAL_CHARS:
        scores.append(-float(len(toks)))
        toks.append(ch)
        types.append(NORMAL)
    for t, s in (("ab", -999.0), ("abc", -1000.0), ("he", -1001.0), ("llo", -1002.0), ("ll", -1003.0),
                 ("lo", -1004.0)):
        toks.append(t)
        types.append(NORMAL)
        scores.append(s)
    merges = "a b\nab c\nh e\nl l\nl o\nll o\n"
    return toks, scores, types, merges


@pytest.fixture(scope="module")
def tok():
    t, s, ty, m = fixture_vocab()
    return BpeTokenizer.from_gguf(t, s, ty, m, TokenizerConfig(bos_token_id=1, eos_token_id=2, unk_token_id=0))


def test_token_types(tok):
    assert tok.token_type(0) == CONTROL and tok.token_type(3) == BYTE and tok.token_type(3 + 256) == NORMAL
    t = BpeTokenizer.from_gguf(["a", "b"], [], [99, 4])
    assert t.token_type(0) == 1 and t.token_type(1) == 4  # TokenType::from(99) = Unknown


def test_empty_tokenizer():
    t = BpeTokenizer.from_gguf([])
    assert t.vocab_size() == 0 and t.bos_token() is None and t.eos_token() is None


def test_encode_basic(tok):
    ids = tok.encode("hi", False)
    assert len(ids) >= 2 and all(i < tok.vocab_size() for i in ids)
    assert tok.decode(ids) == "hi"


def test_encode_with_bos_eos():
    t, s, ty, m = fixture_vocab()
    k = BpeTokenizer.from_gguf(t, s, ty, m, TokenizerConfig(bos_token_id=1, eos_token_id=2, prepend_bos=True,
                                                              add_eos=True))
    ids = k.encode("hi", True)
    assert ids[0] == 1 and ids[-1] == 2 and len(ids) > 2
    assert k.encode("hi", False)[0] != 1


def test_decode_and_roundtrip(tok):
    for text in ["abc", "hello", "hi there", "Hello, World!", "a", "test 123"]:
        assert tok.decode(tok.encode(text, False)) == text, text


def test_byte_fallback(tok):
    for b in range(256):
        i = tok.byte_token(b)
        assert i != 0 and i < tok.vocab_size() and tok.token_to_piece(i) == f"<0x{b:02X}>"
    # '1', '2', '3' are not in the vocabulary: their UTF-8 bytes
    ids = tok.encode("123", False)
    assert [tok.token_to_piece(i) for i in ids] == ["<0x31>", "<0x32>", "<0x33>"]


def test_bpe_merges(tok):
    ids = tok.encode("abc", False)
    assert [tok.token_to_piece(i) for i in ids] == ["abc"]
    ids = tok.encode("hello", False)
    assert [tok.token_to_piece(i) for i in ids] == ["he", "llo"]
    assert [tok.token_to_piece(i) for i in tok.encode("ab", False)] == ["ab"]


def test_vocab_size_and_pieces(tok):
    assert tok.vocab_size() == 3 + 256 + len(NORMAL_CHARS) + 6
    assert tok.token_to_piece(1) == "<s>" and tok.token_to_piece(10 ** 6) is None


def test_from_gguf_basic():
    t = BpeTokenizer.from_gguf(["<s>", "</s>"], [0.0, 0.0], [3, 3], None,
                               TokenizerConfig(bos_token_id=0, eos_token_id=1))
    assert t.vocab_size() == 2 and t.bos_token() == 0 and t.eos_token() == 1


def test_pretokenizer_leftmost_first(tok):
    # ' ?[^\s]+' keeps one leading space; '\s+' takes a whole run; "'s" only
    # where a piece starts; space runs stay one piece
    pieces = lambda s: [tok.decode([i]) for i in tok.encode(s, False)]  # noqa: E731
    assert "".join(pieces("a  b")) == "a  b"
    assert tok.decode(tok.encode("it's a test", False)) == "it's a test"
    assert tok.decode(tok.encode("\tab \n", False)) == "\tab \n"


def test_encode_with_special(tok):
    ids = tok.encode_with_special("<s>hello</s>ab")
    assert ids[0] == 1 and 2 in ids
    assert tok.decode(ids) == "<s>hello</s>ab"


def _kv_str_array(key, items):
    return gstr(key) + struct.pack("<IIQ", ARR, STR, len(items)) + b"".join(gstr(x) for x in items)


def _kv_f32_array(key, items):
    return gstr(key) + struct.pack("<IIQ", ARR, F32, len(items)) + struct.pack(f"<{len(items)}f", *items)


def _kv_i32_array(key, items):
    return gstr(key) + struct.pack("<IIQ", ARR, I32, len(items)) + struct.pack(f"<{len(items)}i", *items)


def test_tokenizer_from_gguf_file(tmp_path):
    """parse_tokenizer_config_from_gguf (src/tokenizer.rs:520-553) on typed
    GGUF keys and the token arrays, read by this library's GGUF parser"""
    t, s, ty, m = fixture_vocab()
    kvs = [_kv_str_array("tokenizer.ggml.tokens", t), _kv_f32_array("tokenizer.ggml.scores", s),
           _kv_i32_array("tokenizer.ggml.token_type", ty),
           _kv_str_array("tokenizer.ggml.merges", [ln for ln in m.splitlines()]),
           gstr("tokenizer.ggml.bos_token_id") + struct.pack("<II", U32, 1),
           gstr("tokenizer.ggml.eos_token_id") + struct.pack("<II", U32, 2),
           gstr("tokenizer.ggml.add_bos") + struct.pack("<IB", BOOL, 1),
           gstr("tokenizer.ggml.add_space_prefix") + struct.pack("<IB", BOOL, 1)]
    data = header(0, len(kvs)) + b"".join(kvs)
    p = tmp_path / "tok.gguf"
    p.write_bytes(data)
    k = BpeTokenizer.from_gguf_file(str(p))
    c = k.config
    assert (c.bos_token_id, c.eos_token_id, c.add_bos, c.add_eos, c.add_space_prefix, c.prepend_bos) == \
        (1, 2, True, False, True, False)
    assert k.vocab_size() == len(t)
    # add_space_prefix: " hello" -> the space, then he + llo
    assert [k.token_to_piece(i) for i in k.encode("hello", False)] == [" ", "he", "llo"]
