// LoRA weight gradients of the frozen projection (lora_down lives in
// fl_lora_down.cu):
//
//   lora_grad : out(p, j) (+)= sum_m P[m, p] * Lo[m, j]          (fp32 out)
//               dA = Us^T . X  (P = X),  dB = dY^T . Ts (P = dY)
//   (reference: the FP32 autograd of F.linear(F.linear(x.float(), A), B),
//   training/recompute.py:102-127)
//
// A skinny reduction over tokens that streams one large BF16 activation once,
// on the warp-level BF16 tensor-core path (mma.sync m16n8k16, fp32
// accumulate); movmatrix turns row-major activation tiles into the transposed
// fragments the reduction over tokens needs.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// hi = bf16(x), lo = bf16(x - hi): packed pairs for two consecutive elements.
__device__ __forceinline__ void split_pair(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(x0, x1);
  const float h0 = __uint_as_float(hi << 16), h1 = __uint_as_float(hi & 0xFFFF0000u);
  lo = pack_bf16x2(x0 - h0, x1 - h1);
}

// ---------------------------------------------------------------- lora_grad
// Warp tile: 32 output rows p x 8*JT columns j, reducing over an M-slice in
// steps of 16 tokens.  Thread (g, c) loads P[m0+g (+8)][p0 + 8c .. 8c+7]; word
// w of that vector is the mma fragment of 8x8 block w whose logical column
// pair c maps to actual p = p0 + 8c + 2w.  movmatrix transposes the blocks into
// A fragments (rows p, k = tokens); logical row g' of block w is actual
// p = p0 + 8(g'/2) + 2w + (g'%2).  Blocks (0,1) form p-tile 0, (2,3) p-tile 1.
template <int JT>
__global__ void __launch_bounds__(128) lora_grad_kernel(const __nv_bfloat16* __restrict__ P, int M, int Pdim,
                                                        const __nv_bfloat16* __restrict__ Q, int rank,
                                                        float* __restrict__ out, int64_t o_sp, int64_t o_sj,
                                                        int m_per_cta, const int4* __restrict__ tiles,
                                                        const int* __restrict__ tile_count,
                                                        int64_t out_expert_stride) {
  __shared__ float red[4][32][8 * JT + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int p0 = blockIdx.x * 32;
  int mbeg = blockIdx.y * m_per_cta;
  int mend = min(M, mbeg + m_per_cta);
  if (tiles != nullptr) {
    // MoE: one token slice of one expert; its gradient is that expert's.
    if (static_cast<int>(blockIdx.y) >= *tile_count) return;
    const int4 t = tiles[blockIdx.y];
    mbeg = t.y;
    mend = t.z;
    out += t.x * out_expert_stride;
  }
  float acc[2][JT][4];
#pragma unroll
  for (int pt = 0; pt < 2; ++pt)
#pragma unroll
    for (int t = 0; t < JT; ++t) acc[pt][t][0] = acc[pt][t][1] = acc[pt][t][2] = acc[pt][t][3] = 0.f;
  const uint4 zero4 = make_uint4(0, 0, 0, 0);
  for (int m = mbeg + warp * 16; m < mend; m += 64) {
    const int ma = m + g, mb = m + g + 8;
    const uint4 xa = ma < mend ? __ldg(reinterpret_cast<const uint4*>(P + static_cast<size_t>(ma) * Pdim + p0 + 8 * c)) : zero4;
    const uint4 xb = mb < mend ? __ldg(reinterpret_cast<const uint4*>(P + static_cast<size_t>(mb) * Pdim + p0 + 8 * c)) : zero4;
    // A fragments: block w of rows g (tokens 0-7) -> a0/a1 (k 0-7); rows g+8 -> a2/a3 (k 8-15).
    const uint32_t ta0 = movmatrix_trans(xa.x), ta1 = movmatrix_trans(xa.y);
    const uint32_t ta2 = movmatrix_trans(xa.z), ta3 = movmatrix_trans(xa.w);
    const uint32_t tb0 = movmatrix_trans(xb.x), tb1 = movmatrix_trans(xb.y);
    const uint32_t tb2 = movmatrix_trans(xb.z), tb3 = movmatrix_trans(xb.w);
#pragma unroll
    for (int t = 0; t < JT; ++t) {
      // B fragment: Q[m + k][t*8 + n] with pairs along k -> transpose 8x8 blocks.
      const uint32_t qa = ma < mend ? __ldg(reinterpret_cast<const uint32_t*>(Q + static_cast<size_t>(ma) * 64 + t * 8 + 2 * c)) : 0u;
      const uint32_t qb = mb < mend ? __ldg(reinterpret_cast<const uint32_t*>(Q + static_cast<size_t>(mb) * 64 + t * 8 + 2 * c)) : 0u;
      const uint32_t b0 = movmatrix_trans(qa), b1 = movmatrix_trans(qb);
      mma_bf16_16816(acc[0][t], ta0, ta1, tb0, tb1, b0, b1);
      mma_bf16_16816(acc[1][t], ta2, ta3, tb2, tb3, b0, b1);
    }
  }
  // Logical tile row -> actual p offset inside the 32-wide warp tile.
#pragma unroll
  for (int pt = 0; pt < 2; ++pt) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int w = 2 * pt + half;  // block index
      const int pr = 8 * (g >> 1) + 2 * w + (g & 1);
#pragma unroll
      for (int t = 0; t < JT; ++t) {
        red[warp][pr][t * 8 + 2 * c] = acc[pt][t][2 * half];
        red[warp][pr][t * 8 + 2 * c + 1] = acc[pt][t][2 * half + 1];
      }
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 32 * 8 * JT; idx += 128) {
    const int pr = idx / (8 * JT), j = idx % (8 * JT);
    const int p = p0 + pr;
    if (j >= rank || p >= Pdim) continue;
    const float v = red[0][pr][j] + red[1][pr][j] + red[2][pr][j] + red[3][pr][j];
    atomicAdd(out + p * o_sp + j * o_sj, v);
  }
}

int launch_lora_grad(const void* P, int M, int Pdim, const void* Q, int rank, float* out, int64_t o_sp,
                     int64_t o_sj, int accumulate, cudaStream_t stream, const int4* tiles, const int* tile_count,
                     int max_tiles, int64_t out_expert_stride, int64_t out_total) {
  if (Pdim % 32 != 0) return set_error(FL_ERR_ARG, "lora_grad: dim %d not a multiple of 32", Pdim);
  if (!accumulate) {
    // out is a dense [Pdim, rank] or [rank, Pdim] fp32 matrix (per expert).
    const size_t n = tiles ? static_cast<size_t>(out_total) : static_cast<size_t>(Pdim) * rank;
    cudaError_t e = cudaMemsetAsync(out, 0, n * sizeof(float), stream);
    if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "lora_grad memset: %s", cudaGetErrorString(e));
  }
  const int ptiles = Pdim / 32;
  int splits = (4 * 148 + ptiles - 1) / ptiles;
  const int max_splits = (M + 63) / 64;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  int m_per_cta = (M + splits - 1) / splits;
  m_per_cta = (m_per_cta + 63) / 64 * 64;
  splits = (M + m_per_cta - 1) / m_per_cta;
  if (tiles) splits = max_tiles;
  if (splits < 1) return FL_OK;
  dim3 grid(ptiles, splits);
  auto p = static_cast<const __nv_bfloat16*>(P);
  auto qq = static_cast<const __nv_bfloat16*>(Q);
  if (rank <= 16)
    lora_grad_kernel<2><<<grid, 128, 0, stream>>>(p, M, Pdim, qq, rank, out, o_sp, o_sj, m_per_cta, tiles,
                                                         tile_count, out_expert_stride);
  else if (rank <= 32)
    lora_grad_kernel<4><<<grid, 128, 0, stream>>>(p, M, Pdim, qq, rank, out, o_sp, o_sj, m_per_cta, tiles,
                                                         tile_count, out_expert_stride);
  else
    lora_grad_kernel<8><<<grid, 128, 0, stream>>>(p, M, Pdim, qq, rank, out, o_sp, o_sj, m_per_cta, tiles,
                                                         tile_count, out_expert_stride);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "lora_grad launch: %s", cudaGetErrorString(e));
  return FL_OK;
}

}  // namespace fl
