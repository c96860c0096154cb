// Standalone group-128 dequantization into a BF16 buffer — the bit-exact
// counterpart of the reference's decode_into (quantization/codecs.py:158-170):
//   out[i] = bf16_rne( fp32(lut[code_i]) * scales[i / 128] )
// with code_i the low nibble of payload[i/2] for even i and the high nibble for
// odd i.  It serves the reference-format slot decode path and the
// bit-exactness tests; the GEMM kernels decode the same way on the fly.
//
// HBM-bound: each thread turns one 32-bit payload word (8 codes) into one
// 16-byte output vector; a warp covers 256 consecutive elements.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {

__global__ void __launch_bounds__(256) dequant_kernel(const uint32_t* __restrict__ payload,
                                                      const float* __restrict__ scales,
                                                      const float* __restrict__ lut, int64_t numel,
                                                      __nv_bfloat16* __restrict__ out, int vec_ok) {
  __shared__ float lut_s[16];
  if (threadIdx.x < 16) lut_s[threadIdx.x] = lut[threadIdx.x];
  __syncthreads();
  const int64_t nwords = (numel + 7) / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < nwords; w += stride) {
    const uint32_t codes = __ldg(payload + w);
    const float s = __ldg(scales + (w >> 4));  // 16 words = 128 elements per group
    uint32_t v[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float lo = __fmul_rn(lut_s[(codes >> (8 * p)) & 15u], s);
      const float hi = __fmul_rn(lut_s[(codes >> (8 * p + 4)) & 15u], s);
      v[p] = pack_bf16x2(lo, hi);
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

int launch_dequant(const uint8_t* payload, const float* scales, const float* lut, int64_t numel, void* out,
                   cudaStream_t stream) {
  if (numel <= 0) return FL_OK;
  if (reinterpret_cast<uintptr_t>(payload) % 4 != 0)
    return set_error(FL_ERR_ARG, "dequant: payload must be 4-byte aligned");
  const int vec_ok = reinterpret_cast<uintptr_t>(out) % 16 == 0;
  const int64_t nwords = (numel + 7) / 8;
  int64_t blocks = (nwords + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  dequant_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(reinterpret_cast<const uint32_t*>(payload), scales,
                                                               lut, numel, static_cast<__nv_bfloat16*>(out),
                                                               vec_ok);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "dequant launch: %s", cudaGetErrorString(e));
  return FL_OK;
}

}  // namespace fl
