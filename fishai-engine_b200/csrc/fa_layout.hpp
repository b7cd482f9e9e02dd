// Device weight layout ("chunked row groups"), shared by host and device.
//
// A GGUF projection W is read by the reference as W[K][N] with N contiguous
// (tensor::matmul, src/tensor.rs:244-258), so its quant blocks run along N.
// On the device each weight is split into column chunks of width <= CW; a
// chunk stores its rows in groups of 8 consecutive rows.  One group holds
// exactly the native bytes of those 8 rows x w columns (no byte is added or
// re-quantised), regrouped so that "lane" j of a warp finds the codes of its
// 32 columns [32j, 32j+32) as one contiguous 16-byte (4-bit types) or 32-byte
// (Q8_0) run, and the group size is a multiple of 16 bytes:
//
//   Q4_0 (blk 32):  codes  r*w/2 + 16j     (byte i: col i low nibble, col i+16 high nibble)
//                   d      4w + (r*w/32 + j)*2               f16
//   Q4_1 (blk 32):  codes  as Q4_0;  d 4w + (r*w/32 + j)*2,  m 4w + w/2 + (r*w/32 + j)*2   f16
//   Q5_0 (blk 32):  low 4 bits as the Q4_0 codes;  qh 4w + (r*w/32 + j)*4 (u32, bit i = col i's
//                   fifth bit, as stored);  d 5w + (r*w/32 + j)*2   f16
//   Q8_0 (blk 32):  codes  r*w + 32j       (byte i: col i, int8)
//                   d      8w + (r*w/32 + j)*2               f16
//   Q4_K (blk 256): codes  r*w/2 + 16j     (as Q4_0)
//                   header 4w + (r*w/256 + s)*16             native d, dmin, scales[12]
//   Q6_K (blk 256): ql     r*w/2 + 16j     (low 4 bits, as Q4_0)
//                   qh     4w + r*w/4 + 8j (byte i: cols i, i+8, i+16, i+24 at bits 0-1,2-3,4-5,6-7)
//                   scales 6w + r*w/16 + 2j   int8, cols [0,16) then [16,32)
//                   d      8*(13w/16) + (r*w/256 + s)*2      f16
//   F16:            r*2w + 64j ;   F32:  r*4w + 128j
//
// (r = row within the group, s = super-block within the row, j = 32-column
// lane.)  Group bytes = 8 x native row bytes, a multiple of 16, so every
// range of whole groups can be moved with one 1-D bulk TMA copy.
#pragma once
#include <stdint.h>

#ifndef FA_HD
#ifdef __CUDACC__
#define FA_HD __host__ __device__
#else
#define FA_HD
#endif
#endif

namespace fa {

enum : int { kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ4_1 = 3, kQ5_0 = 6, kQ8_0 = 8, kQ4_K = 12, kQ6_K = 14 };

// bytes of one row of `w` columns in native GGML blocks.  A Q4_K row of
// w = 256 s + 128 columns (a tensor-parallel shard holding half of a
// super-block) is stored as s + 1 whole blocks, the half block re-encoded as
// a block whose upper 128 columns are zero (tp_shard_columns).
FA_HD inline uint32_t native_row_bytes(int type, uint32_t w) {
  switch (type) {
    case kF32: return 4 * w;
    case kF16: return 2 * w;
    case kQ4_0: return w / 32 * 18;
    case kQ4_1: return w / 32 * 20;
    case kQ5_0: return w / 32 * 22;
    case kQ8_0: return w / 32 * 34;
    case kQ4_K: return (w + 255) / 256 * 144;
    case kQ6_K: return w / 256 * 210;
    default: return 0;
  }
}
FA_HD inline uint32_t group_bytes(int type, uint32_t w) { return 8 * native_row_bytes(type, w); }
FA_HD inline uint32_t type_block(int type) {
  return (type == kQ4_K || type == kQ6_K) ? 256u : (type == kF32 || type == kF16) ? 1u : 32u;
}
FA_HD inline bool gemv_type_supported(int type) {
  return type == kF32 || type == kF16 || type == kQ4_0 || type == kQ4_1 || type == kQ5_0 || type == kQ8_0 ||
         type == kQ4_K || type == kQ6_K;
}

// ---------------------------------------------------------------------------
// Tensor-core layout ("MMA tiles") for Q4_K, Q6_K, Q8_0 and Q4_0.
//
// A chunk of width w is stored as groups of 16 consecutive rows; a group
// holds exactly the native bytes of those rows (16 * native_row_bytes).  The
// codes are re-ordered for mma.sync.m16n8k16 with the weight as operand A:
// A[m][k] = code of (row k, column m) of a 16 x 16 tile, so one tile is one
// MMA.  Columns are cut into 64-wide slices (4 tiles; the last slice of a
// chunk may hold 2 tiles) and lane l = 4g + c of a warp holds, per tile, the
// eight fragment elements e = 0..7 at (m, k) = (g + 8*((e>>1)&1),
// 2c + (e&1) + 8*(e>>2)).
//
//   Q4_K / Q4_0 codes:  slice i at 512 i, lane l at + 4 nt l, tile t at + 4t:
//                       one u32 per tile, element e at bit 4(e>>1) + 16(e&1)
//   Q6_K  low 4 bits:   as the Q4 codes (region 0, 8w bytes)
//         high 2 bits:  region 8w: slice i at 256 i, lane l at + 8 l; word
//                       h (tiles 2h, 2h+1), element e of tile t at bit
//                       4(e>>1) + 16(e&1) + 2(t&1)
//   Q8_0 codes (q+128): slice i at 1024 i, lane l at + 8 nt l, tile t at + 8t:
//                       two u32, element e in word e>>2, byte 2(e&1) + ((e>>1)&1)
//   Q4_K header:        region 8w, (super-block s, row r) at (16 s + r) * 16:
//                       d, dmin, then the 12 scale bytes re-laid as eight
//                       12-bit fields (sc | m << 6), field f at bit 12f
//   Q6_K scales:        region 12w, int8 (16-col sub-block j, row r) at 16 j + r
//        d:             region 13w, f16 (super-block s, row r) at (16 s + r) * 2
//   Q8_0 / Q4_0 d:      region 16w / 8w, f16 (32-col block b, row r) at (16 b + r) * 2
//
// (nt = tiles in the slice.)  Q4_0 keeps its codes 0..15 (value d(q-8)), Q8_0
// stores q+128 in 0..255 (value d(u-128)): the same information, re-encoded.
// ---------------------------------------------------------------------------
FA_HD inline bool mma_type(int type) { return type == kQ4_K || type == kQ6_K || type == kQ8_0 || type == kQ4_0; }
// a Q4_K group holds 8w code bytes and one 16-byte header per row and
// super-block (so a half super-block takes 8w + 256 bytes, no padding)
FA_HD inline uint32_t mma_group_bytes(int type, uint32_t w) {
  return type == kQ4_K ? 8 * w + 256 * ((w + 255) / 256) : 16 * native_row_bytes(type, w);
}
// row m / column k of fragment element e of lane l inside a 16x16 tile
FA_HD inline uint32_t frag_m(uint32_t l, uint32_t e) { return l / 4 + 8 * ((e >> 1) & 1); }
FA_HD inline uint32_t frag_k(uint32_t l, uint32_t e) { return 2 * (l % 4) + (e & 1) + 8 * (e >> 2); }
FA_HD inline uint32_t frag_q4_bit(uint32_t e) { return 4 * (e >> 1) + 16 * (e & 1); }
FA_HD inline uint32_t frag_q8_byte(uint32_t e) { return 4 * (e >> 2) + 2 * (e & 1) + ((e >> 1) & 1); }

// One column chunk of a GEMV launch.  All chunks of a launch share K.
struct ChunkDesc {
  uint64_t offset;   // byte offset of the chunk's first row group in the weight buffer
  uint32_t gbytes;   // bytes per row group (8 rows; 16 in the MMA layout)
  uint16_t type;     // ggml type
  uint16_t width;    // columns (multiple of 32; of 256 for K-quants)
  uint32_t out_col;  // first output column of the chunk in the launch's output space
  uint32_t contrib_off;  // first entry of this chunk in the launch's contributor list
  uint32_t n_contrib;    // CTAs that contribute partial sums to this chunk
  uint32_t sgroups;      // row groups per pipeline stage (k_gemv_mma)
};

// Contiguous range of (chunk, row group) units streamed by one CTA:
// from (c0, g0) inclusive to (c1, g1) exclusive, chunk-major order.
struct CtaRange {
  uint32_t c0, g0, c1, g1;
};

}  // namespace fa
