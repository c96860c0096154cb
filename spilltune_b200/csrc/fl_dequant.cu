// Standalone group-128 dequantization into a BF16 buffer — the bit-exact
// counterpart of the reference's decode_into (quantization/codecs.py:158-170):
//   out[i] = bf16_rne( fp32(lut[code_i]) * scales[i / 128] )
// with code_i the low nibble of payload[i/2] for even i and the high nibble for
// odd i.  It serves the reference-format slot decode path and the
// bit-exactness tests; the GEMM kernels decode the same way on the fly.  The
// same kernel decodes the bitsandbytes NF4-DQ64 layout (layout 1: even element
// in the high nibble, one scale per 64 elements from the DQ prologue below).
//
// HBM-bound: each thread turns one 32-bit payload word (8 codes) into one
// 16-byte output vector; a warp covers 256 consecutive elements.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_codebook.cuh"
#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {

template <int kLayout>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ payload,
                                                      const float* __restrict__ scales,
                                                      const float* __restrict__ lut, int64_t numel,
                                                      __nv_bfloat16* __restrict__ out, int vec_ok) {
  __shared__ float lut_s[16];
  if (threadIdx.x < 16) lut_s[threadIdx.x] = lut[threadIdx.x];
  __syncthreads();
  const int64_t nwords = (numel + 7) / 8;
  const int64_t nbytes = kLayout == kLayoutG128 ? nwords * 4 : (numel + 1) / 2;  // DQ64 packs exactly
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < nwords; w += stride) {
    uint32_t codes;
    if (4 * w + 4 <= nbytes) {
      codes = __ldg(reinterpret_cast<const uint32_t*>(payload) + w);
    } else {  // ragged last word of a DQ64 record: only its own bytes exist
      codes = 0;
      for (int b = 0; b < 4 && 4 * w + b < nbytes; ++b) codes |= static_cast<uint32_t>(__ldg(payload + 4 * w + b)) << (8 * b);
    }
    // 16 words = 128 elements per group (layout 0), 8 words = 64 per block (layout 1)
    const float s = __ldg(scales + (kLayout == kLayoutG128 ? (w >> 4) : (w >> 3)));
    uint32_t v[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t c_even = kLayout == kLayoutG128 ? (codes >> (8 * p)) & 15u : (codes >> (8 * p + 4)) & 15u;
      const uint32_t c_odd = kLayout == kLayoutG128 ? (codes >> (8 * p + 4)) & 15u : (codes >> (8 * p)) & 15u;
      v[p] = pack_bf16x2(__fmul_rn(lut_s[c_even], s), __fmul_rn(lut_s[c_odd], s));
    }
    const int64_t e0 = w * 8;
    if (vec_ok && e0 + 8 <= numel) {
      *reinterpret_cast<uint4*>(out + e0) = make_uint4(v[0], v[1], v[2], v[3]);
    } else {
      for (int e = 0; e < 8 && e0 + e < numel; ++e) {
        const uint16_t bits = static_cast<uint16_t>((v[e >> 1] >> (16 * (e & 1))) & 0xFFFFu);
        reinterpret_cast<uint16_t*>(out)[e0 + e] = bits;
      }
    }
  }
}

// Double-quantization prologue of a DQ64 record: FP32 block scales
//   a[b] = fp32(nested_map[absmax_q[b]] * nested_absmax[b / 256]) + offset
// (two separately rounded operations, no fused multiply-add).
__global__ void __launch_bounds__(256) nf4dq_prologue_kernel(const uint8_t* __restrict__ absmax_q,
                                                             const float* __restrict__ nested_absmax,
                                                             const float* __restrict__ nested_map, float offset,
                                                             int64_t blocks, float* __restrict__ out) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < blocks; b += stride)
    out[b] = __fadd_rn(__fmul_rn(__ldg(nested_map + __ldg(absmax_q + b)), __ldg(nested_absmax + (b >> 8))), offset);
}

int launch_nf4dq_prologue(const uint8_t* absmax_q, const float* nested_absmax, const float* nested_map, float offset,
                          int64_t blocks, float* out, cudaStream_t stream) {
  if (blocks <= 0) return FL_OK;
  int64_t grid = (blocks + 255) / 256;
  if (grid > 148 * 8) grid = 148 * 8;
  nf4dq_prologue_kernel<<<static_cast<int>(grid), 256, 0, stream>>>(absmax_q, nested_absmax, nested_map, offset,
                                                                    blocks, out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "nf4dq prologue launch: %s", cudaGetErrorString(e));
  return FL_OK;
}

int launch_dequant(const uint8_t* payload, const float* scales, const float* lut, int64_t numel, void* out,
                   cudaStream_t stream, int layout) {
  if (numel <= 0) return FL_OK;
  if (reinterpret_cast<uintptr_t>(payload) % 4 != 0)
    return set_error(FL_ERR_ARG, "dequant: payload must be 4-byte aligned");
  const int vec_ok = reinterpret_cast<uintptr_t>(out) % 16 == 0;
  const int64_t nwords = (numel + 7) / 8;
  int64_t blocks = (nwords + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (layout == kLayoutG128)
    dequant_kernel<kLayoutG128><<<static_cast<int>(blocks), 256, 0, stream>>>(payload, scales, lut, numel,
                                                                             static_cast<__nv_bfloat16*>(out), vec_ok);
  else
    dequant_kernel<kLayoutNf4Dq64><<<static_cast<int>(blocks), 256, 0, stream>>>(
        payload, scales, lut, numel, static_cast<__nv_bfloat16*>(out), vec_ok);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "dequant launch: %s", cudaGetErrorString(e));
  return FL_OK;
}

}  // namespace fl
