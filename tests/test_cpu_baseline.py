"""CPU-only checks of the measurement plumbing:

* the oracle's copy of the synthetic GGUF writer (oracle/build/libsynth.so,
  which the CPU reference arm of bench.py uses so that it never loads the
  CUDA library) writes files byte-identical to the library's fa_synth_write
  (no GPU is needed for either);
* the whole-token reference-order timing (or_time_token) computes the same
  token as the oracle's forward on the same cache, so what it times is the
  reference's forward and not a shortcut."""
import hashlib
import os

import numpy as np

import oracle as O
from fishai_engine import synth


def _sha(p):
    return hashlib.sha256(open(p, "rb").read()).hexdigest()


def test_oracle_writer_is_byte_identical(tmp_path):
    for name, over in (("tiny-q8_0", {}), ("llama3-8b-q4_k_m", dict(n_layers=1, vocab=2048, n_ff=1024, n_embd=512,
                                                                       n_heads=4, n_kv_heads=2)),
                       ("llama2-7b-q4_0", dict(n_layers=1, vocab=1024, n_ff=512, n_embd=256, n_heads=4,
                                               n_kv_heads=4))):
        a = synth.write_preset(name, str(tmp_path / "a.gguf"), **over)
        b = synth.write_preset(name, str(tmp_path / "b.gguf"), writer=O.write_gguf, **over)
        assert _sha(a) == _sha(b), name


def test_time_token_computes_the_reference_forward(tmp_path):
    p = synth.write_preset("tiny-q8_0", str(tmp_path / "t.gguf"), writer=O.write_gguf)
    m = O.Model(p, threads=os.cpu_count() or 2)
    for n_cached, tok in ((0, 5), (40, 1234)):
        kv_t, kv_f = m.kv(64), m.kv(64)
        kv_t.fill_synthetic(n_cached, seed=3)
        kv_f.fill_synthetic(n_cached, seed=3)
        ls, hs, picked = m.time_token(kv_t, tok, n_cached, 0)
        logits = m.forward([tok], n_cached, kv_f, algo=0)
        assert picked == int(np.argmax(logits))
        assert len(kv_t) == len(kv_f) == n_cached + 1
        assert ls > 0 and hs > 0
