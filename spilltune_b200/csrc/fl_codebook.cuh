// Codebook decode helpers shared by every kernel that turns packed 4-bit
// group-128 codes into BF16 operands.
//
// Decode rule (ram_vram_finetune/quantization/codecs.py:158-170, generalised to
// a 16-entry FP32 codebook): w = bf16_rne( fp32(lut[c]) * fp32(scale[group]) ).
// The reference int4-sym-g128 format is lut[c] = c - 8; NF4 uses the NF4 table.
// Codes are packed two per byte, the even element in the low nibble.
#pragma once
#include "fl_ptx.cuh"

namespace fl {

// Per-(row, group) table of the 16 possible BF16 products, split into a
// low-byte plane and a high-byte plane so that prmt can look up four codes at a
// time.  Building it costs 16 FP32 multiplies; each product is rounded exactly
// once, so every looked-up value equals the element-wise decode bit for bit.
struct ProductTable {
  uint32_t lo[4];  // byte c of the plane = low byte of bf16(lut[c]*scale)
  uint32_t hi[4];  // byte c of the plane = high byte
};

__device__ __forceinline__ ProductTable make_table(const float (&lut)[16], float scale) {
  uint32_t p[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) p[i] = pack_bf16x2(__fmul_rn(lut[2 * i], scale), __fmul_rn(lut[2 * i + 1], scale));
  ProductTable t;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    t.lo[i] = prmt(p[2 * i], p[2 * i + 1], 0x6420);
    t.hi[i] = prmt(p[2 * i], p[2 * i + 1], 0x7531);
  }
  return t;
}

// Decode the four codes held in nibbles 0..3 of `w16` (bits 0..15) into two
// bf16x2 words: out0 = {e0 (low half), e1}, out1 = {e2, e3}.
__device__ __forceinline__ void lookup4(const ProductTable& t, uint32_t w16, uint32_t& out0, uint32_t& out1) {
  const uint32_t sel = w16 & 0x7777u;                 // low 3 bits of each code
  const uint32_t mask = prmt(w16 << 4, w16, 0xD9C8);  // 0xFF per byte where code bit 3 is set
  const uint32_t lo = (prmt(t.lo[0], t.lo[1], sel) & ~mask) | (prmt(t.lo[2], t.lo[3], sel) & mask);
  const uint32_t hi = (prmt(t.hi[0], t.hi[1], sel) & ~mask) | (prmt(t.hi[2], t.hi[3], sel) & mask);
  out0 = prmt(lo, hi, 0x5140);
  out1 = prmt(lo, hi, 0x7362);
}

// Eight codes of one 32-bit payload word -> four bf16x2 words in element order.
__device__ __forceinline__ void lookup8(const ProductTable& t, uint32_t w, uint32_t* out) {
  lookup4(t, w & 0xFFFFu, out[0], out[1]);
  lookup4(t, w >> 16, out[2], out[3]);
}

}  // namespace fl
