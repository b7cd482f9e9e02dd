"""Exactness of the packed-f16 Q8_0 / Q4_0 dequantisation of the token GEMM.

The tensor-core GEMM turns a Q8_0 or Q4_0 code into its f16 A-operand value
in packed half arithmetic (fishai-engine_b200/csrc/qgemm.cu, deq_pairs_q0):
the code goes into the mantissa of 1024.0 (f16 0x6400 | code == 1024 + code),
one subtraction of 1024 + z leaves code - z, one multiplication by the row
scale d rounds.  The K-quant path instead computes d * code - d * z in f32
and rounds that to f16.  These tests check, for every code and a wide range
of f16 scales (subnormals included), that both give the same f16 bits (up
to the sign of a zero), i.e. that the packed path equals the exact product
d * (code - z) rounded once to f16 (the Q8_0 value of src/quant.rs:261-290
and the Q4_0 value of src/quant.rs:123-157, the stored code offset by z).

numpy evaluates float16 arithmetic in float32 and rounds the result once to
float16; a product or difference of two f16 values is exact in float32, so
that is the IEEE f16 result the GPU's HSUB2 / HMUL2 produce.
"""
import numpy as np
import pytest


def _scales():
    rng = np.random.default_rng(7)
    bits = rng.integers(0, 0x7C00, 20000, dtype=np.uint16)  # finite positive f16, subnormals included
    d = bits.view(np.float16)
    d = np.concatenate([d, -d, np.array([0.0, 2.0**-24, 2.0**-14, 1.0, 65504.0 / 256.0], np.float16)])
    return d[np.isfinite(d)]


def _f32_path(d, codes, z):
    # d * code - d * z in f32 (both products exact), rounded once to f16
    d32 = d.astype(np.float32)[:, None]
    c32 = codes.astype(np.float32)[None, :]
    v = d32 * c32 - d32 * np.float32(z)
    with np.errstate(over="ignore"):
        return v.astype(np.float16)


def _packed_path(d, codes, z):
    h = (np.uint16(0x6400) | codes.astype(np.uint16)).view(np.float16)  # 1024 + code, exactly
    assert np.array_equal(h.astype(np.float32), 1024.0 + codes.astype(np.float32))
    q = h - np.float16(1024 + z)  # code - z, exact in f16
    assert np.array_equal(q.astype(np.float32), codes.astype(np.float32) - z)
    with np.errstate(over="ignore"):
        return (q[None, :] * d[:, None]).astype(np.float16)


@pytest.mark.parametrize("ncodes,z", [(256, 128), (16, 8)], ids=["q8_0", "q4_0"])
def test_packed_f16_matches_f32_rounding(ncodes, z):
    d = _scales()
    codes = np.arange(ncodes, dtype=np.uint32)
    ref = _f32_path(d, codes, z)
    got = _packed_path(d, codes, z)
    finite = np.isfinite(ref.astype(np.float32))
    # same bits wherever the value is representable (beyond 65504 both overflow
    # to inf), except the sign of a zero: code == z with d < 0 is +0 in f32
    # (x - x) and -0 in f16 (0 * d), equal values that add the same to the
    # GEMM's f32 accumulators
    zero = ref.astype(np.float32) == 0.0
    assert np.array_equal(got.astype(np.float32)[zero], ref.astype(np.float32)[zero])
    keep = finite & ~zero
    assert np.array_equal(ref.view(np.uint16)[keep], got.view(np.uint16)[keep])
    assert np.array_equal(np.isinf(ref), np.isinf(got))
