// Host quantisers used by the synthetic GGUF writer.
//  Q8_0, Q4_0: the reference crate's own rules (src/quant.rs:393-471):
//    d = max|x|/127 (resp. /8), stored as f16, codes round(x/d) with the
//    unrounded f32 d; Q4_0 packs element 2j in the HIGH nibble of byte j.
//  Q4_1, Q5_0: this library's encoders for the reference's layouts
//    (src/quant.rs:163-255), element 2j in the high nibble of byte j.
//  Q4_K, Q6_K: this library's encoders for the public GGUF block layouts
//    (any valid encoding works: the oracle and the device read the same file).
#pragma once
#include <cstddef>
#include <cstdint>

namespace fa {
// n must be a multiple of the block size; returns bytes written
size_t quantize_row(int ggml_type, const float *x, size_t n, uint8_t *out);
}  // namespace fa
