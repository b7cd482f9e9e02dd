"""Token-parallel dequant-GEMM (tcgen05, f16 operands, f32 accumulation)
against the oracle's dequantised weights: Y = f16(X) . f16(W) in f64.
The only differences left are the f32 accumulation order and a rare 1-ulp
f16 rounding difference of a weight, so the bar is 1e-3 of max |Y|."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from fishai_engine import _lib as L
from fishai_engine import synth
from fishai_engine.model import ModelWeights

pytestmark = pytest.mark.gpu


def f16(a):
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float64)


def _w(g, name):
    i = g.tensor_info(name)
    ne0, ne1 = (i["dims"] + [1])[:2]
    return O.dequantize(g.read_tensor_data(name), i["ggml_type"], ne0 * ne1).reshape(ne1, ne0)


def _launch_weight(g, proj, layer):
    """W[K][n_out] in the launch output space of the weight group"""
    b = f"blk.{layer}."
    if proj == 0:
        return np.concatenate([_w(g, b + "attn_q.weight"), _w(g, b + "attn_k.weight"), _w(g, b + "attn_v.weight")], 1)
    if proj == 1:
        return _w(g, b + "attn_output.weight")
    if proj == 2:  # gate and up interleaved per 1024-column chunk
        gt, up = _w(g, b + "ffn_gate.weight"), _w(g, b + "ffn_up.weight")
        F, cols = gt.shape[1], []
        for c0 in range(0, 2 * F, 1024):
            w = min(1024, 2 * F - c0)
            g0 = c0 // 2
            cols += [gt[:, g0:g0 + w // 2], up[:, g0:g0 + w // 2]]
        return np.concatenate(cols, 1)
    if proj == 3:
        return _w(g, b + "ffn_down.weight")
    return _w(g, "output.weight")


def _gemm(dev, proj, layer, x):
    T, n = x.shape[0], C.c_uint32()
    L.check(L.lib().fa_gemm_tokens(dev._h, proj, layer, L.f32_ptr(x), T, None, C.byref(n)))
    y = np.zeros((T, n.value), np.float32)
    L.check(L.lib().fa_gemm_tokens(dev._h, proj, layer, L.f32_ptr(x), T, L.f32_ptr(y), C.byref(n)))
    return y


def _kq_spec(**kw):
    spec = dict(n_layers=2, n_embd=512, n_heads=8, n_kv_heads=4, n_ff=1536, vocab=4096, context_len=256,
                rope_base=500000.0, norm_eps=1e-5, sigma=0.02, type_embd=O.Q4_K, type_q=O.Q4_K, type_k=O.Q4_K,
                type_v=O.Q6_K, type_o=O.Q4_K, type_gate=O.Q4_K, type_up=O.Q4_K, type_down=O.Q6_K, type_out=O.Q6_K)
    spec.update(kw)
    return spec


MODELS = {
    "q8_0": None,
    "q4k_q6k": _kq_spec(),
    "q4_0": _kq_spec(type_embd=O.Q4_0, type_q=O.Q4_0, type_k=O.Q4_0, type_v=O.Q4_0, type_o=O.Q4_0,
                     type_gate=O.Q4_0, type_up=O.Q4_0, type_down=O.Q4_0, type_out=O.Q6_K, n_kv_heads=8),
    # mixed-type launches (qkv: Q8_0, Q4_0 and Q6_K chunks) load the weights
    # directly; single-type Q8_0 / Q4_0 launches go through the prefetch ring
    "mixed": _kq_spec(type_q=O.Q8_0, type_k=O.Q4_0, type_v=O.Q6_K, type_o=O.Q8_0, type_gate=O.Q4_0,
                      type_up=O.Q4_0, type_down=O.Q8_0, type_out=O.Q8_0),
}


@pytest.fixture(scope="module", params=list(MODELS))
def model(request, tmp_path_factory):
    path = str(tmp_path_factory.mktemp("qg") / f"{request.param}.gguf")
    spec = MODELS[request.param]
    p = synth.write_preset("tiny-q8_0", path) if spec is None else synth.write(path, 9, **spec)
    dev = ModelWeights.load_from_gguf(p)
    yield dev, O.GGUF(p)
    dev.close()


@pytest.mark.parametrize("proj", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("T", [1, 37, 64, 130, 300])
def test_token_gemm_matches_dequantised_weights(model, proj, T):
    dev, g = model
    layer = 1 if proj != 4 else 0
    W = _launch_weight(g, proj, layer)
    x = np.random.default_rng(proj * 1000 + T).normal(0.0, 1.0, (T, W.shape[0])).astype(np.float32)
    y = _gemm(dev, proj, layer, x)
    assert y.shape == (T, W.shape[1])
    ref = f16(x) @ f16(W)
    err = np.max(np.abs(y - ref)) / np.max(np.abs(ref))
    assert err <= 1e-3, err
