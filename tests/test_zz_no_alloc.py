"""fa_sdpa_noalloc — attention for callers that cannot allocate device memory
(their memory comes from their own pool, or cudaMalloc is off limits on their
latency path).  It keeps its scratch in a fixed static device array inside the
library.  Checked through the C ABI against fa_sdpa, the allocating entry
point with the same arguments, on two calls in a row (the second reuses the
array the first left behind).  Tolerance: max-abs-rel <= 1e-5, as for fa_sdpa.

Named to be collected last, so that a run stopping at its first failure has
run every other test before this one."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _mar(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _call(name, q, k, v, q_len, kv_len, H, KVH, hd, out):
    import torch
    from fishai_engine import _lib as L

    stream = torch.cuda.current_stream().cuda_stream
    return getattr(L.lib(), name)(q.data_ptr(), k.data_ptr(), v.data_ptr(), q_len, kv_len, H, KVH, hd,
                                  out.data_ptr(), stream)


def test_noalloc_matches_fa_sdpa_twice():
    import torch
    from fishai_engine import _lib as L

    # first call larger than the second: the second must not depend on what
    # the first left in the shared array
    cases = [(3, 500, 32, 8, 128, 11), (1, 2049, 8, 2, 64, 12)]
    for q_len, kv_len, H, KVH, hd, seed in cases:
        g = torch.Generator().manual_seed(seed)
        q = torch.randn(q_len, H * hd, generator=g).cuda()
        k = torch.randn(kv_len, KVH * hd, generator=g).cuda()
        v = torch.randn(kv_len, KVH * hd, generator=g).cuda()
        want = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        L.check(_call("fa_sdpa", q, k, v, q_len, kv_len, H, KVH, hd, want))
        L.check(_call("fa_sdpa_noalloc", q, k, v, q_len, kv_len, H, KVH, hd, got))
        torch.cuda.synchronize()
        got, want = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(got).all()
        assert _mar(got, want) <= 1e-5


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import torch
    from fishai_engine import _lib as L

    # head_dim 128: q_len * n_heads * 32 * 130 floats must fit in 524288
    q_len, kv_len, H, KVH, hd = 4, 8, 32, 8, 128
    q = torch.zeros(q_len, H * hd, device="cuda")
    k = torch.zeros(kv_len, KVH * hd, device="cuda")
    out = torch.zeros_like(q)
    rc = _call("fa_sdpa_noalloc", q, k, k, q_len, kv_len, H, KVH, hd, out)
    assert rc == L.ERR_INVALID
    assert "exceeds the fixed scratch" in L.last_error()


def test_noalloc_allocates_no_device_memory():
    """After one warm call, a call with a larger shape than any before it
    leaves the device's free memory unchanged (fa_sdpa, by contrast, grows its
    scratch for such a call)."""
    import torch
    from fishai_engine import _lib as L

    def run(q_len, kv_len, H, KVH, hd):
        q = torch.ones(q_len, H * hd, device="cuda")
        k = torch.ones(kv_len, KVH * hd, device="cuda")
        out = torch.empty_like(q)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        L.check(_call("fa_sdpa_noalloc", q, k, k, q_len, kv_len, H, KVH, hd, out))
        torch.cuda.synchronize()
        return free0, torch.cuda.mem_get_info()[0]

    run(1, 16, 4, 4, 64)  # warm: symbol lookup, module load
    before, after = run(3, 4096, 32, 8, 128)  # larger than any call so far
    assert before == after


def test_noalloc_rejects_too_many_query_rows_per_kv_head():
    """the second limit: q_len * n_kv_heads <= 1024 (here 129 * 8 = 1032
    while the partials, 129 * 8 * 32 * 4 floats, would still fit)"""
    import torch
    from fishai_engine import _lib as L

    q_len, kv_len, H, KVH, hd = 129, 4, 8, 8, 2
    q = torch.zeros(q_len, H * hd, device="cuda")
    k = torch.zeros(kv_len, KVH * hd, device="cuda")
    out = torch.zeros_like(q)
    rc = _call("fa_sdpa_noalloc", q, k, k, q_len, kv_len, H, KVH, hd, out)
    assert rc == L.ERR_INVALID
    assert "q_len*n_kv_heads = 1032" in L.last_error()
