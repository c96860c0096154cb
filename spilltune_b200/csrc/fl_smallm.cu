// Small-M frozen projection (M <= 16 tokens: decode-like steps):
//
//   Y[m, n] = sum_g scale[n, g] * sum_{k in g} X[m, k] * L[code[n, k]]  +  sum_j Ts[m, j] * Blora[n, j]
//
// the same product as fl_fwd with each 128-wide scale group factored out of
// its dot product, so the tensor-core operand is L = bf16(lut) — exactly the
// stored code for int4-sym (c - 8), the bf16-rounded codebook for NF4 — and the
// scale multiplies the fp32 partial sum of its group.
//
// At M <= 16 every weight byte is used once, so the kernel is bound by HBM
// reads of the packed weights (0.53 B per weight).  Decoding must therefore be
// cheap: a 256-entry table maps one payload byte (two codes) to a bf16 pair,
// stored once per lane in shared memory (entry e of lane l at word e*32 + l, so
// a warp's lookups never conflict); one prmt + one IMAD + one shared load per
// two weights.  The MMAs are warp-level (mma.sync m16n8k16): a warp owns 32
// weight rows as the A operand (rows g and g+8 of each 16-row tile) and the
// tokens are the 8-wide N dimension.  The reduction dimension is split over a
// cluster of CTAs whose partial sums meet in rank 0's shared memory
// (distributed shared memory), which also adds the LoRA term and writes Y.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {
namespace sm {

constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kRowsPerWarp = 32;                 // two 16-row MMA tiles
constexpr int kRows = kWarps * kRowsPerWarp;     // 128 rows per CTA
constexpr int kLutBytes = 256 * 32 * 4;          // per-lane byte -> bf16x2 table
constexpr int kRing = 3;                         // groups of codes in flight per thread
constexpr int kRingBytes = kRing * kThreads * 80;  // per thread per group: 4 x 16 B codes + 4 x 4 B scales

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bf16 pair for the two codes of byte `pos` of `w`, from this lane's table.
__device__ __forceinline__ uint32_t lut_pair(const uint32_t* lut_lane, uint32_t w, uint32_t pos) {
  const uint32_t byte = prmt(w, 0u, 0x4440u | pos);
  return lut_lane[byte * 32];
}

template <int NT>  // 8-token tiles: 1 (M <= 8) or 2 (M <= 16)
__global__ void __launch_bounds__(kThreads)
    smallm_kernel(const __nv_bfloat16* __restrict__ X, const __nv_bfloat16* __restrict__ Ts,
                  const uint8_t* __restrict__ codes, const float* __restrict__ scales, const float* __restrict__ lut,
                  const float* __restrict__ blora, int rank, __nv_bfloat16* __restrict__ Y, int M, int N, int K,
                  int split) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* lut_s = reinterpret_cast<uint32_t*>(smem);                       // kLutBytes
  const int groups = K / 128;
  const uint32_t crank = cluster_ctarank();
  const int g_begin = static_cast<int>(crank) * groups / split;
  const int g_end = (static_cast<int>(crank) + 1) * groups / split;
  const int ks = (g_end - g_begin) * 128;                                   // this CTA's reduction slice
  const int ks_pad = (groups + split - 1) / split * 128 + 8;                // row stride of the X slice
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem + kLutBytes);  // [8*NT][ks_pad]
  float* red = reinterpret_cast<float*>(smem + kLutBytes + 8 * NT * ks_pad * 2);  // [split-1][kRows][8*NT]
  uint8_t* ring = smem + kLutBytes + 8 * NT * ks_pad * 2 + (split - 1) * kRows * 8 * NT * 4;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c4 = lane & 3;
  const int n0 = (blockIdx.x / split) * kRows;

  // Per-lane table: entry e = {bf16(lut[e & 15]) (low half), bf16(lut[e >> 4])}.
  for (int e = warp; e < 256; e += kWarps)
    lut_s[e * 32 + lane] = pack_bf16x2(__ldg(lut + (e & 15)), __ldg(lut + (e >> 4)));
  // X slice: tokens 0..8*NT-1 (zero past M), reduction columns of this CTA.
  for (int idx = threadIdx.x; idx < 8 * NT * (ks / 8); idx += kThreads) {
    const int t = idx / (ks / 8), c = idx % (ks / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < M) v = __ldg(reinterpret_cast<const uint4*>(X + static_cast<size_t>(t) * K + g_begin * 128 + 8 * c));
    *reinterpret_cast<uint4*>(xs + t * ks_pad + 8 * c) = v;
  }
  __syncthreads();

  const uint32_t* lut_lane = lut_s + lane;
  float acc[2][NT][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[t][nt][0] = acc[t][nt][1] = acc[t][nt][2] = acc[t][nt][3] = 0.f;

  // Rows this thread feeds: tile t, half h -> n0 + 32*warp + 16*t + g + 8*h.
  int rows[2][2];
  bool rvalid[2][2];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rows[t][h] = n0 + kRowsPerWarp * warp + 16 * t + g + 8 * h;
      rvalid[t][h] = rows[t][h] < N;
    }
  const size_t row_bytes = static_cast<size_t>(K) / 2;

  // Ring slot of group gi for this thread: 4 code segments then 4 scales.
  auto slot = [&](int gi) { return ring + ((gi % kRing) * kThreads + threadIdx.x) * 80; };
  auto issue = [&](int gi) {
    if (gi < g_end) {
      uint8_t* d = slot(gi);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const bool v = rvalid[t][h];
          const int r = v ? rows[t][h] : 0;
          cp_async_16(d + (2 * t + h) * 16, codes + r * row_bytes + gi * 64 + 16 * c4, v);
          cp_async_4(d + 64 + (2 * t + h) * 4, scales + static_cast<size_t>(r) * groups + gi, v);
        }
    }
    cp_async_commit();  // one group per call, empty past the end, so wait counts stay uniform
  };
#pragma unroll
  for (int a = 0; a < kRing - 1; ++a) issue(g_begin + a);

  uint4 q[2][2];
  float sc[2][2];
  for (int gi = g_begin; gi < g_end; ++gi) {
    issue(gi + kRing - 1);
    cp_async_wait<kRing - 1>();
    {
      const uint8_t* d = slot(gi);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          q[t][h] = *reinterpret_cast<const uint4*>(d + (2 * t + h) * 16);
          sc[t][h] = *reinterpret_cast<const float*>(d + 64 + (2 * t + h) * 4);
        }
    }
    float part[2][NT][4];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) part[t][nt][0] = part[t][nt][1] = part[t][nt][2] = part[t][nt][3] = 0.f;
    // MMA k-step kk uses bytes 2kk (k = 32c4+4kk+{0,1}) and 2kk+1 (+{2,3}) of the thread's 16 bytes.
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int col = (gi - g_begin) * 128 + 32 * c4 + 4 * kk;
      uint32_t b[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint2 bv = *reinterpret_cast<const uint2*>(xs + (8 * nt + g) * ks_pad + col);
        b[nt][0] = bv.x;
        b[nt][1] = bv.y;
      }
      const uint32_t wsel = kk >> 1;             // word of the 16-byte chunk
      const uint32_t p0 = 2 * (kk & 1), p1 = p0 + 1;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const uint32_t w0 = wsel == 0 ? q[t][0].x : wsel == 1 ? q[t][0].y : wsel == 2 ? q[t][0].z : q[t][0].w;
        const uint32_t w1 = wsel == 0 ? q[t][1].x : wsel == 1 ? q[t][1].y : wsel == 2 ? q[t][1].z : q[t][1].w;
        const uint32_t a0 = lut_pair(lut_lane, w0, p0), a1 = lut_pair(lut_lane, w1, p0);
        const uint32_t a2 = lut_pair(lut_lane, w0, p1), a3 = lut_pair(lut_lane, w1, p1);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816(part[t][nt], a0, a1, a2, a3, b[nt][0], b[nt][1]);
      }
    }
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        acc[t][nt][0] = fmaf(sc[t][0], part[t][nt][0], acc[t][nt][0]);
        acc[t][nt][1] = fmaf(sc[t][0], part[t][nt][1], acc[t][nt][1]);
        acc[t][nt][2] = fmaf(sc[t][1], part[t][nt][2], acc[t][nt][2]);
        acc[t][nt][3] = fmaf(sc[t][1], part[t][nt][3], acc[t][nt][3]);
      }
  }
  cp_async_wait<0>();

  // ------------------------------------------------------------ cluster reduction
  // Accumulator element i of tile t / token tile nt: row rows[t][i / 2],
  // token 8*nt + 2*c4 + (i & 1).  Slot within the CTA: (local row, token).
  cluster_sync();  // every CTA is past its reads of X / the table; rank 0's `red` is free
  if (crank != 0) {
    const uint32_t base = mapa_shared(smem_u32(red), 0) + static_cast<uint32_t>((crank - 1) * kRows * 8 * NT * 4);
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int lr = kRowsPerWarp * warp + 16 * t + g + 8 * (i >> 1);
          const int tok = 8 * nt + 2 * c4 + (i & 1);
          st_shared_cluster_u32(base + (lr * 8 * NT + tok) * 4, __float_as_uint(acc[t][nt][i]));
        }
  }
  cluster_sync();
  if (crank == 0) {
    // LoRA operands for the epilogue, staged once in areas the main loop is
    // done with: Ts rows of the tokens in the X slice (>= 8*NT*136 bf16), the
    // CTA's Blora rows in the 32 KiB byte table (kRows x rank <= 64 floats).
    float* ts_s = reinterpret_cast<float*>(xs);                   // [8*NT][64]
    float* b_s = reinterpret_cast<float*>(lut_s);                 // [kRows][rank]
    if (rank > 0) {
      for (int idx = threadIdx.x; idx < 8 * NT * 64; idx += kThreads) {
        const int tok = idx >> 6, j = idx & 63;
        ts_s[idx] = (tok < M && j < rank) ? __bfloat162float(Ts[static_cast<size_t>(tok) * 64 + j]) : 0.f;
      }
      for (int idx = threadIdx.x; idx < kRows * rank; idx += kThreads) {
        const int lr = idx / rank;
        b_s[idx] = (n0 + lr < N) ? __ldg(blora + static_cast<size_t>(n0) * rank + idx) : 0.f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int lr = kRowsPerWarp * warp + 16 * t + g + 8 * (i >> 1);
          const int tok = 8 * nt + 2 * c4 + (i & 1);
          float v = acc[t][nt][i];
          for (int p = 0; p < split - 1; ++p) v += red[(p * kRows + lr) * 8 * NT + tok];
          const int n = n0 + lr;
          if (n < N && tok < M) {
            const float* tr = ts_s + tok * 64;
            const float* br = b_s + lr * rank;
            for (int j = 0; j < rank; ++j) v = fmaf(tr[j], br[j], v);
            Y[static_cast<size_t>(tok) * N + n] = __float2bfloat16_rn(v);
          }
        }
  }
}

template <int NT>
static int launch_nt(const void* X, const void* Ts, const uint8_t* codes, const float* scales, const float* lut,
                     const float* blora, int rank, void* Y, int M, int N, int K, int split, cudaStream_t stream) {
  const int groups = K / 128;
  const int ks_pad = (groups + split - 1) / split * 128 + 8;
  const size_t smem = kLutBytes + static_cast<size_t>(8 * NT) * ks_pad * 2 +
                      static_cast<size_t>(split - 1) * kRows * 8 * NT * 4 + kRingBytes;
  if (smem > 227 * 1024) return set_error(FL_ERR_UNSUPPORTED, "small-M path: K=%d too large", K);
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&smallm_kernel<NT>),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "small-M attr: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(split * ((N + kRows - 1) / kRows));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t le = cudaLaunchKernelEx(&cfg, smallm_kernel<NT>, static_cast<const __nv_bfloat16*>(X),
                                      static_cast<const __nv_bfloat16*>(Ts), codes, scales, lut, blora, rank,
                                      static_cast<__nv_bfloat16*>(Y), M, N, K, split);
  if (le != cudaSuccess) return set_error(FL_ERR_CUDA, "small-M launch: %s", cudaGetErrorString(le));
  return FL_OK;
}

}  // namespace sm

int launch_smallm_fwd(const void* X, const void* Ts, const uint8_t* codes, const float* scales, const float* lut,
                      const float* lora, int rank, void* Y, int M, int N, int K, cudaStream_t stream) {
  if (M < 1 || M > 16) return set_error(FL_ERR_ARG, "small-M path needs 1 <= M <= 16");
  if (K % 128 != 0) return set_error(FL_ERR_ARG, "small-M path needs K %% 128 == 0");
  // Enough CTAs to cover the SMs twice; a cluster holds at most 8.
  const int row_tiles = (N + sm::kRows - 1) / sm::kRows;
  int split = (2 * 148 + row_tiles - 1) / row_tiles;
  if (split > 4) split = 4;  // clusters of <= 4 keep several clusters resident per GPC
  if (split > K / 128) split = K / 128;
  if (split < 1) split = 1;
  // Keep the X slice + partials within shared memory.
  auto bytes = [&](int sp) {
    return sm::kLutBytes + 16LL * ((K / 128 + sp - 1) / sp * 128 + 8) * 2 + (sp - 1) * sm::kRows * 16LL * 4 +
           sm::kRingBytes;
  };
  while (split > 1 && bytes(split) > 220 * 1024) --split;
  while (split < 8 && bytes(split) > 220 * 1024) ++split;
  if (M <= 8) return sm::launch_nt<1>(X, Ts, codes, scales, lut, lora, rank, Y, M, N, K, split, stream);
  return sm::launch_nt<2>(X, Ts, codes, scales, lut, lora, rank, Y, M, N, K, split, stream);
}

}  // namespace fl
