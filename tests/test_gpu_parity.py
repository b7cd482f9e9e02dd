"""Parity of the sm_100a path (through the C ABI) against the oracle, the C
restatement of the reference CPU path.  Tolerances (the project's parity
criteria): dequantised blocks bit-exact; hidden states and logits
max-abs-rel <= 1e-4 on the f32 path; greedy ids identical."""
import os

import numpy as np
import pytest

import oracle as O
from fishai_engine import _lib as L
from fishai_engine import synth
from fishai_engine.model import ModelWeights, GenerationConfig, GenerationState

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-4


def max_abs_rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.fixture(scope="module")
def tmpdir_m(tmp_path_factory):
    return tmp_path_factory.mktemp("gpu")


def _rand_blocks(rng, t, nblocks):
    bs = O.type_size(t)
    raw = rng.integers(0, 256, size=(nblocks, bs), dtype=np.uint8)
    # sane f16 scales: exponent field away from inf/nan
    def f16s(n, lo=-8, hi=2):
        v = (rng.uniform(0.5, 1.0, n) * 2.0 ** rng.integers(lo, hi, n)).astype(np.float16)
        return v.view(np.uint8).reshape(n, 2)
    if t in (O.Q4_0, O.Q8_0, O.Q5_0):
        raw[:, 0:2] = f16s(nblocks)
    elif t == O.Q4_1:
        raw[:, 0:2] = f16s(nblocks)
        raw[:, 2:4] = f16s(nblocks)
    elif t == O.Q4_K:
        raw[:, 0:2] = f16s(nblocks)
        raw[:, 2:4] = f16s(nblocks)
    elif t == O.Q6_K:
        raw[:, 208:210] = f16s(nblocks)
    elif t == O.F16:
        raw[:] = f16s(nblocks, -14, 15)
    elif t == O.F32:
        raw = rng.normal(0, 1, nblocks).astype(np.float32).view(np.uint8).reshape(nblocks, 4)
    return raw.reshape(-1)


@pytest.mark.parametrize("t", [O.F32, O.F16, O.Q4_0, O.Q4_1, O.Q5_0, O.Q8_0, O.Q4_K, O.Q6_K])
def test_dequant_bit_exact(t):
    from fishai_engine.quant import dequantize
    rng = np.random.default_rng(t)
    nb = 777
    raw = _rand_blocks(rng, t, nb)
    count = nb * O.block_size(t)
    dev = dequantize(raw, t, count)
    ref = O.dequantize(raw, t, count)
    assert dev.size == ref.size == count
    assert np.array_equal(dev.view(np.uint32), ref.view(np.uint32))


def test_dequant_short_data_truncates():
    from fishai_engine.quant import dequantize
    raw = _rand_blocks(np.random.default_rng(1), O.Q8_0, 3)[: 34 * 2 + 5]
    assert dequantize(raw, O.Q8_0, 96).size == 64


def _model_pair(path, resident=False, step=False):
    dev = ModelWeights.load_from_gguf(path, use_step_kernel=step)
    assert dev.step_kernel_active == step
    return dev, O.Model(path, resident=resident, threads=os.cpu_count() or 4)


def _forward_parity(path, n_tokens=6, kv_dtype=L.KV_F32, check_hidden=True, seed=0, step=False, fixed=False):
    dev, ref = _model_pair(path, step=step)
    if fixed:  # split-K pieces summed in a fixed order instead of red.add
        L.check(L.lib().fa_debug_set(dev._h, L.DEBUG_FIXED_ORDER_SUMS, 1))
    V = dev.config.vocab_size
    rng = np.random.default_rng(seed)
    toks = rng.integers(3, V, n_tokens).tolist()
    kv_d = dev.new_kv_cache(64, dtype=kv_dtype)
    kv_r = ref.kv(64, kv_f16=kv_dtype == L.KV_F16)
    worst = 0.0
    for i, t in enumerate(toks):
        # a hidden-state dump runs the per-kernel step, so the step kernel is checked on logits and cache
        if check_hidden:
            lg_d, am_d, hid_d = dev.forward([t], i, kv_d, return_argmax=True, hidden=True)
        else:
            lg_d, am_d = dev.forward([t], i, kv_d, return_argmax=True)
        lg_r, hid_r = ref.forward([t], i, kv_r, algo=1, hidden=True)
        worst = max(worst, max_abs_rel(lg_d, lg_r))
        if check_hidden:
            for l in range(dev.config.n_layers):
                assert max_abs_rel(hid_d[l, 0], hid_r[l, 0]) <= TOL_F32, (i, l)
        assert max_abs_rel(lg_d, lg_r) <= TOL_F32, i
        assert int(am_d[0]) == int(np.argmax(lg_d))
    return worst, dev, ref, kv_d, kv_r


def test_tiny_q8_0_forward_parity(tmpdir_m):
    p = synth.write_preset("tiny-q8_0", str(tmpdir_m / "tiny.gguf"))
    worst, dev, ref, kv_d, kv_r = _forward_parity(p)
    # KVCache::get parity
    for layer in (0, dev.config.n_layers - 1):
        kd, vd = kv_d.get(layer)
        kr, vr = kv_r.get(layer)
        assert max_abs_rel(kd, kr) <= TOL_F32 and max_abs_rel(vd, vr) <= TOL_F32


def _kquant_spec(**kw):
    spec = dict(n_layers=2, n_embd=512, n_heads=8, n_kv_heads=4, n_ff=1536, vocab=4096, context_len=256,
                rope_base=500000.0, norm_eps=1e-5, sigma=0.02, type_embd=O.Q4_K, type_q=O.Q4_K, type_k=O.Q4_K,
                type_v=O.Q6_K, type_o=O.Q4_K, type_gate=O.Q4_K, type_up=O.Q4_K, type_down=O.Q6_K, type_out=O.Q6_K)
    spec.update(kw)
    return spec


def test_kquant_mix_forward_parity(tmpdir_m):
    p = synth.write(str(tmpdir_m / "kq.gguf"), 7, **_kquant_spec())
    _forward_parity(p)


def test_kquant_mix_fixed_order_sums_parity(tmpdir_m):
    """The fixed-order split-K reduction (last arriver per chunk) at the same
    bars as the default red.add one, and bit-reproducible: the same token
    stepped twice from the same cache state gives identical logits."""
    p = synth.write(str(tmpdir_m / "kq_fixed.gguf"), 7, **_kquant_spec())
    _, dev, _, kv_d, _ = _forward_parity(p, fixed=True, check_hidden=False)
    a = dev.forward([17], 6, kv_d)
    kv2 = dev.new_kv_cache(64, dtype=L.KV_F32)
    toks = [int(x) for x in np.random.default_rng(0).integers(3, dev.config.vocab_size, 6)]
    for i, t in enumerate(toks):
        dev.forward([t], i, kv2)
    b = dev.forward([17], 6, kv2)
    assert np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


def test_q4_0_forward_parity(tmpdir_m):
    p = synth.write(str(tmpdir_m / "q40.gguf"), 1, **_kquant_spec(
        type_embd=O.Q4_0, type_q=O.Q4_0, type_k=O.Q4_0, type_v=O.Q4_0, type_o=O.Q4_0, type_gate=O.Q4_0,
        type_up=O.Q4_0, type_down=O.Q4_0, type_out=O.Q6_K, n_kv_heads=8, rope_base=10000.0))
    _forward_parity(p)


def test_q4_1_q5_0_forward_parity(tmpdir_m):
    """Q4_1 (q*d + m) and Q5_0 ((q-16)*d, fifth bit in qh) projections, the
    reference's other block types (src/quant.rs:163-255), mixed in one model
    (the CUDA-core GEMV's 8-row layout) with a Q8_0 head; hidden states and
    logits at the f32 bar, then 12 greedy ids equal to the oracle's."""
    p = synth.write(str(tmpdir_m / "q41q50.gguf"), 5, **_kquant_spec(
        n_embd=256, n_heads=4, n_kv_heads=2, n_ff=512, vocab=2048, type_embd=O.Q4_1, type_q=O.Q4_1, type_k=O.Q5_0,
        type_v=O.Q4_1, type_o=O.Q5_0, type_gate=O.Q4_1, type_up=O.Q4_1, type_down=O.Q5_0, type_out=O.Q8_0,
        rope_base=10000.0))
    _, dev, ref, _, _ = _forward_parity(p)
    prompt = [5, 77, 1024, 9]
    cfg = GenerationConfig(max_tokens=16, temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=1.0)
    assert GenerationState(dev, cfg).generate(prompt) == ref.generate(prompt, 16, fast=True).tolist()


def test_f16_f32_tied_forward_parity(tmpdir_m):
    p = synth.write(str(tmpdir_m / "f.gguf"), 3, **_kquant_spec(
        n_embd=256, n_heads=4, n_kv_heads=2, n_ff=640, vocab=1000, type_embd=O.F16, type_q=O.F16, type_k=O.F32,
        type_v=O.F16, type_o=O.F32, type_gate=O.F16, type_up=O.F16, type_down=O.F32, type_out=-1))
    _forward_parity(p)


def test_f16_kv_cache_parity(tmpdir_m):
    # device f16 cache against the oracle with f16-rounded K/V
    p = synth.write_preset("tiny-q8_0", str(tmpdir_m / "tiny16.gguf"))
    _forward_parity(p, kv_dtype=L.KV_F16, check_hidden=False)


# the persistent step kernel (one launch per token): same bars as the per-kernel path
@pytest.mark.parametrize("name,spec", [
    ("tiny", None),                                            # Q8_0, 4 q heads per kv head
    ("kq", dict()),                                            # Q4_K / Q6_K mix, 2 per kv head
    ("q40", dict(type_embd=O.Q4_0, type_q=O.Q4_0, type_k=O.Q4_0, type_v=O.Q4_0, type_o=O.Q4_0, type_gate=O.Q4_0,
                 type_up=O.Q4_0, type_down=O.Q4_0, type_out=O.Q6_K, n_kv_heads=8, rope_base=10000.0)),  # MHA
    ("mq8", dict(n_kv_heads=1, type_k=O.Q8_0, type_v=O.Q8_0)),  # 8 per kv head
])
def test_step_kernel_forward_parity(tmpdir_m, name, spec):
    path = str(tmpdir_m / f"step_{name}.gguf")
    p = synth.write_preset("tiny-q8_0", path) if spec is None else synth.write(path, 5, **_kquant_spec(**spec))
    worst, dev, ref, kv_d, kv_r = _forward_parity(p, n_tokens=8, check_hidden=False, step=True)
    for layer in (0, dev.config.n_layers - 1):
        kd, vd = kv_d.get(layer)
        kr, vr = kv_r.get(layer)
        assert max_abs_rel(kd, kr) <= TOL_F32 and max_abs_rel(vd, vr) <= TOL_F32


def test_step_kernel_f16_kv_parity(tmpdir_m):
    p = synth.write_preset("tiny-q8_0", str(tmpdir_m / "step16.gguf"))
    _forward_parity(p, kv_dtype=L.KV_F16, check_hidden=False, step=True)


def test_step_kernel_greedy_generate_matches_oracle(tmpdir_m):
    p = synth.write_preset("tiny-q8_0", str(tmpdir_m / "stepg.gguf"))
    dev, ref = _model_pair(p, step=True)
    prompt = np.random.default_rng(1).integers(3, 32000, 40).tolist()
    n_gen = 96
    st = GenerationState(dev, GenerationConfig(max_tokens=40 + n_gen, temperature=0.0, top_k=0, top_p=1.0,
                                               repetition_penalty=1.0))
    assert st.generate(prompt) == ref.generate(prompt, 40 + n_gen, fast=True).tolist()


def test_compat_multi_token_forward(tmpdir_m):
    """forward(&[a,b,c], pos): same RoPE position, no mask (src/model.rs:367-394)"""
    p = synth.write_preset("tiny-q8_0", str(tmpdir_m / "tinyc.gguf"))
    dev, ref = _model_pair(p)
    kv_d, kv_r = dev.new_kv_cache(32), ref.kv(32)
    dev.forward([11], 0, kv_d)
    ref.forward([11], 0, kv_r, algo=1)
    lg_d, hid_d = dev.forward([7, 900, 31000], 1, kv_d, hidden=True)
    lg_r, hid_r = ref.forward([7, 900, 31000], 1, kv_r, algo=1, hidden=True)
    assert max_abs_rel(lg_d, lg_r) <= TOL_F32
    assert max_abs_rel(hid_d, hid_r) <= TOL_F32
    assert kv_d.seq_len_with_dim(0, kv_d.kv_dim) == 4


def test_prefill_equals_sequential(tmpdir_m):
    p = synth.write_preset("tiny-q8_0", str(tmpdir_m / "tinyp.gguf"))
    dev, ref = _model_pair(p)
    toks = list(range(100, 140))
    kv_a, kv_b = dev.new_kv_cache(64), dev.new_kv_cache(64)
    last, am = dev.prefill(toks, 0, kv_a)
    for i, t in enumerate(toks):
        seq_lg = dev.forward([t], i, kv_b)
    assert max_abs_rel(last, seq_lg) <= 1e-6
    kv_r = ref.kv(64)
    lr, _ = ref.prefill(toks, 0, kv_r)
    assert max_abs_rel(last, lr) <= TOL_F32
    assert am == int(np.argmax(last))


def test_tiny_greedy_generate_matches_oracle(tmpdir_m):
    p = synth.write_preset("tiny-q8_0", str(tmpdir_m / "tinyg.gguf"))
    dev, ref = _model_pair(p)
    prompt = np.random.default_rng(0).integers(3, 32000, 32).tolist()
    n_gen = 128
    st = GenerationState(dev, GenerationConfig(max_tokens=32 + n_gen, temperature=0.0, top_k=0, top_p=1.0,
                                               repetition_penalty=1.0))
    gen = st.generate(prompt)
    want = ref.generate(prompt, 32 + n_gen, fast=True).tolist()
    assert len(gen) == n_gen
    assert gen == want


def test_generate_stop_and_max_tokens(tmpdir_m):
    p = synth.write_preset("tiny-q8_0", str(tmpdir_m / "tinys.gguf"))
    dev, ref = _model_pair(p)
    prompt = [5, 6, 7, 8]
    full = GenerationState(dev, GenerationConfig(max_tokens=12, temperature=0.0, top_k=0, top_p=1.0,
                                                 repetition_penalty=1.0)).generate(prompt)
    assert len(full) == 8
    stop = full[3]
    cut = GenerationState(dev, GenerationConfig(max_tokens=12, temperature=0.0, top_k=0, top_p=1.0,
                                                repetition_penalty=1.0, stop_token_ids=[stop])).generate(prompt)
    assert cut == full[: full.index(stop)]
    assert ref.generate(prompt, 12, stop_ids=[stop], fast=True).tolist() == cut
    # max_tokens <= prompt length: nothing generated (src/model.rs:683-686)
    assert GenerationState(dev, GenerationConfig(max_tokens=3, temperature=0.0, top_k=0, top_p=1.0,
                                                 repetition_penalty=1.0)).generate(prompt) == []


def test_bad_inputs_fail_loudly(tmpdir_m):
    p = synth.write_preset("tiny-q8_0", str(tmpdir_m / "tinye.gguf"))
    dev = ModelWeights.load_from_gguf(p)
    kv = dev.new_kv_cache(4)
    with pytest.raises(L.FishaiError):
        dev.forward([40000], 0, kv)  # token >= vocab
    for i in range(4):
        dev.forward([1], i, kv)
    with pytest.raises(L.FishaiError) as e:
        dev.forward([1], 4, kv)  # cache full
    assert e.value.code == L.ERR_CONTEXT
    with pytest.raises(IndexError):
        kv.get(99)
