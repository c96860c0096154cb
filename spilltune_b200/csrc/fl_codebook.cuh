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

// `lut` may point to shared or global memory (16 floats).
__device__ __forceinline__ ProductTable make_table(const float* lut, float scale) {
  ProductTable t;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 a = *reinterpret_cast<const float4*>(lut + 4 * i);
    const uint32_t p0 = pack_bf16x2(__fmul_rn(a.x, scale), __fmul_rn(a.y, scale));
    const uint32_t p1 = pack_bf16x2(__fmul_rn(a.z, scale), __fmul_rn(a.w, scale));
    t.lo[i] = prmt(p0, p1, 0x6420);
    t.hi[i] = prmt(p0, p1, 0x7531);
  }
  return t;
}

// Look up four codes: `sel` holds their low three bits in nibbles 0..3 (bit 3
// of each nibble clear), `mask` is 0xFF in byte i when code i has bit 3 set.
// Returns two bf16x2 words: out0 = {e0 (low half), e1}, out1 = {e2, e3}.
__device__ __forceinline__ void lookup4(const ProductTable& t, uint32_t sel, uint32_t mask, uint32_t& out0,
                                        uint32_t& out1) {
  const uint32_t lo = (prmt(t.lo[0], t.lo[1], sel) & ~mask) | (prmt(t.lo[2], t.lo[3], sel) & mask);
  const uint32_t hi = (prmt(t.hi[0], t.hi[1], sel) & ~mask) | (prmt(t.hi[2], t.hi[3], sel) & mask);
  out0 = prmt(lo, hi, 0x5140);
  out1 = prmt(lo, hi, 0x7362);
}

// Record layouts the kernels decode (FL_LAYOUT_* in the C header):
//   0  the reference's group-128 record: even element in the low nibble,
//      one FP32 scale per 128 elements;
//   1  bitsandbytes NF4 double-quantized, block 64: even element in the HIGH
//      nibble, one FP32 scale per 64 elements (from the DQ prologue).
constexpr int kLayoutG128 = 0;
constexpr int kLayoutNf4Dq64 = 1;

// As lookup4, for a word whose codes are paired high nibble first: returns
// out0 = {e1 (low half), e0}, out1 = {e3, e2} — the element order of a
// high-nibble-first byte stream.
__device__ __forceinline__ void lookup4_hf(const ProductTable& t, uint32_t sel, uint32_t mask, uint32_t& out0,
                                           uint32_t& out1) {
  const uint32_t lo = (prmt(t.lo[0], t.lo[1], sel) & ~mask) | (prmt(t.lo[2], t.lo[3], sel) & mask);
  const uint32_t hi = (prmt(t.hi[0], t.hi[1], sel) & ~mask) | (prmt(t.hi[2], t.hi[3], sel) & mask);
  out0 = prmt(lo, hi, 0x4051);
  out1 = prmt(lo, hi, 0x6273);
}

// Eight codes of one 32-bit payload word (element i in nibble i) -> four bf16x2
// words in element order.  The selector and bit-3 masks of both halves come
// from one AND, one shift and two prmt (sign-replicate mode): byte i of a mask
// copies the sign of the byte holding bit 3 of code i, either in w or in w<<4.
__device__ __forceinline__ void lookup8(const ProductTable& t, uint32_t w, uint32_t* out) {
  const uint32_t sel = w & 0x77777777u;
  const uint32_t w4 = w << 4;
  const uint32_t mask_lo = prmt(w4, w, 0xD9C8);  // codes 0..3
  const uint32_t mask_hi = prmt(w4, w, 0xFBEA);  // codes 4..7
  lookup4(t, sel, mask_lo, out[0], out[1]);
  lookup4(t, sel >> 16, mask_hi, out[2], out[3]);
}

}  // namespace fl

namespace fl {

// Layout-generic form: four bf16x2 words in element order for either layout.
template <int kLayout>
__device__ __forceinline__ void lookup8_l(const ProductTable& t, uint32_t w, uint32_t* out) {
  if constexpr (kLayout == kLayoutG128) {
    lookup8(t, w, out);
  } else {
    const uint32_t sel = w & 0x77777777u;
    const uint32_t w4 = w << 4;
    const uint32_t mask_lo = prmt(w4, w, 0xD9C8);
    const uint32_t mask_hi = prmt(w4, w, 0xFBEA);
    lookup4_hf(t, sel, mask_lo, out[0], out[1]);
    lookup4_hf(t, sel >> 16, mask_hi, out[2], out[3]);
  }
}

}  // namespace fl
