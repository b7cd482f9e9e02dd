"""fa_sdpa (tensor::scaled_dot_product_attention on the device) against the
oracle and the reference's own known answers (src/tensor.rs:785-827).
Tolerance: f32 path, max-abs-rel <= 1e-5 (only the summation order differs)."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def mar(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))


def test_reference_known_answers():
    from fishai_engine.tensor import scaled_dot_product_attention as sdpa

    out = sdpa([1.0, 0.0], [1.0, 0.0, 0.0, 1.0], [1.0, 0.0, 0.0, 1.0], 1, 2).reshape(-1)
    assert abs(out[0] - 0.67) < 0.05 and abs(out[1] - 0.33) < 0.05


@pytest.mark.parametrize("q_len,kv_len,H,KVH,hd", [(1, 1, 4, 4, 64), (1, 300, 8, 2, 64), (3, 77, 32, 8, 128),
                                                   (1, 2049, 4, 1, 32), (2, 5, 2, 2, 8)])
def test_matches_oracle(q_len, kv_len, H, KVH, hd):
    from fishai_engine.tensor import scaled_dot_product_attention as sdpa

    rng = np.random.default_rng(kv_len)
    q = rng.normal(0, 1, (q_len, H * hd)).astype(np.float32)
    k = rng.normal(0, 1, (kv_len, KVH * hd)).astype(np.float32)
    v = rng.normal(0, 1, (kv_len, KVH * hd)).astype(np.float32)
    got = sdpa(q, k, v, H, hd, KVH).reshape(q_len, H * hd)
    # the reference expands kv heads (src/model.rs:500-526) then runs SDPA
    rep = H // KVH
    ke = np.repeat(k.reshape(kv_len, KVH, hd), rep, axis=1).reshape(kv_len, H * hd)
    ve = np.repeat(v.reshape(kv_len, KVH, hd), rep, axis=1).reshape(kv_len, H * hd)
    want = O.sdpa(q, ke, ve, H, hd).reshape(q_len, H * hd)
    assert mar(got, want) <= 1e-5


def test_device_pointer_form_matches_host_form():
    import torch

    from fishai_engine.tensor import scaled_dot_product_attention as sdpa
    from fishai_engine.tensor import scaled_dot_product_attention_device as sdpa_dev

    rng = np.random.default_rng(7)
    q = rng.normal(0, 1, (2, 8 * 64)).astype(np.float32)
    k = rng.normal(0, 1, (100, 2 * 64)).astype(np.float32)
    v = rng.normal(0, 1, (100, 2 * 64)).astype(np.float32)
    want = sdpa(q, k, v, 8, 64, 2)
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
    od = torch.empty_like(qd)
    sdpa_dev(qd, kd, vd, od, 2, 100, 8, 64, 2, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(od.cpu().numpy(), want)
