// Host-side helpers shared by the C-ABI implementation: error state, f16
// conversion, ggml type table.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <string>

#include "../../include/fishai_cuda.h"

namespace fa {

// thread-local last error (fa_last_error)
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
const std::string &last_error();

// f16 <-> f32 with the half crate's semantics (exact widening, RNE narrowing)
float f16_to_f32(uint16_t h);
uint16_t f32_to_f16(float f);

// ggml block geometry (src/quant.rs:345-382)
size_t block_elems(int type);
size_t block_bytes(int type);
bool type_known(int type);
// bytes of `n` elements of `type` (n a multiple of the block size)
inline size_t type_nbytes(int type, size_t n) { return n / block_elems(type) * block_bytes(type); }

}  // namespace fa
