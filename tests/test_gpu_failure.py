"""Failure paths, made on the host (nothing faults or hangs a GPU):

* a bounded device wait that runs out: the decode GEMV's producer is told to
  withhold its weight copies (fa_debug_set) and the wait limit is shortened to
  2 ms, so every consumer wait expires; the kernel returns, the call reports
  FA_ERR_TIMEOUT, and after the hooks are cleared the same model decodes
  correctly again (checked against the oracle);
* a device allocation that cannot succeed: a KV cache far beyond the GPU's
  memory returns FA_ERR_OOM instead of aborting, and the model keeps working.

The reference has neither path (it runs on the CPU and panics on misuse,
src/http.rs:855-862)."""
import os

import numpy as np
import pytest

import oracle as O
from fishai_engine import _lib as L
from fishai_engine import synth
from fishai_engine.model import ModelWeights

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():
    path = synth.cached_preset("tiny-q8_0")
    dev = ModelWeights.load_from_gguf(path)
    yield path, dev
    dev.close()


def _mar(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / np.max(np.abs(b)))


def test_expired_device_wait_reports_timeout_and_recovers(tiny):
    path, dev = tiny
    lib = L.lib()
    L.check(lib.fa_debug_set(dev._h, L.DEBUG_WAIT_LIMIT_NS, 2_000_000))
    L.check(lib.fa_debug_set(dev._h, L.DEBUG_WITHHOLD_WEIGHTS, 1))
    try:
        kv = dev.new_kv_cache(16)
        with pytest.raises(L.FishaiError) as e:
            dev.forward([7], 0, kv)
        assert e.value.code == L.ERR_TIMEOUT
    finally:
        L.check(lib.fa_debug_set(dev._h, L.DEBUG_WITHHOLD_WEIGHTS, 0))
        L.check(lib.fa_debug_set(dev._h, L.DEBUG_WAIT_LIMIT_NS, 0))
    # the context and the model are intact: a fresh decode matches the oracle
    kv = dev.new_kv_cache(16)
    got = dev.forward([7], 0, kv)
    ref = O.Model(path, threads=os.cpu_count() or 4)
    want = ref.forward([7], 0, ref.kv(16), algo=1)
    assert _mar(got, want) <= 1e-4


def test_unsatisfiable_kv_allocation_reports_oom(tiny):
    path, dev = tiny
    with pytest.raises(L.FishaiError) as e:
        dev.new_kv_cache(4_000_000, n_seq=64)  # ~1 PB of f32 K/V
    assert e.value.code == L.ERR_OOM
    kv = dev.new_kv_cache(16)
    _, am = dev.forward([9], 0, kv, return_argmax=True, want_logits=False)
    assert 0 <= int(am[0]) < dev.config.vocab_size
