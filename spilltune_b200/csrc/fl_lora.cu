// LoRA weight gradients of the frozen projection (lora_down lives in
// fl_lora_down.cu):
//
//   lora_grad : out(p, j) (+)= sum_m P[m, p] * Lo[m, j]          (fp32 out)
//               dA = Us^T . X  (P = X),  dB = dY^T . Ts (P = dY; at rank <= 16
//               lora_down sums dB in its pass over dY instead)
//   (reference: the FP32 autograd of F.linear(F.linear(x.float(), A), B),
//   training/recompute.py:102-127)
//
// A reduction over tokens that streams the large BF16 activation P once.  The
// token index is the MMA's K, while both P and Lo are contiguous along the
// other index, so both operands enter the 5th-gen tensor core MN-major
// straight from TMA tiles (128-byte swizzle): no software transposes.  One CTA
// owns 128 columns p (the TMEM lanes) and one slice of tokens; D[p, j] (64
// TMEM columns, fp32) is added into the gradient with global reductions.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {
namespace lg {

constexpr int kP = 128;                      // p per CTA (TMEM lanes; UMMA M)
constexpr int kJ = 64;                       // Lo columns (UMMA N; rank padded)
constexpr int kStageM = 64;                  // tokens per stage
constexpr int kStages = 4;
constexpr int kPBox = kStageM * 64 * 2;      // 8 KiB: 64 tokens x 64 p
constexpr int kPBytes = 2 * kPBox;           // 16 KiB: two MN atoms of 64 p
constexpr int kQBytes = kStageM * kJ * 2;    // 8 KiB
constexpr int kThreads = 192;                // warp 0 TMA, warp 1 TMEM + MMA, warps 2-5 epilogue
constexpr int kTmemCols = 64;

struct __align__(8) Bars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t accum;
  uint32_t tmem_base;
  uint32_t abort_word;
};

constexpr int kSmemBytes = 1024 + kStages * (kPBytes + kQBytes) + static_cast<int>(sizeof(Bars));

__global__ void __launch_bounds__(kThreads)
    lora_grad_kernel(const __grid_constant__ CUtensorMap tm_p,  // P [M, Pdim] bf16, box {64, 64}
                     const __grid_constant__ CUtensorMap tm_q,  // Lo [M, 64] bf16, box {64, 64}
                     float* __restrict__ out, int64_t o_sp, int64_t o_sj, int rank, int M, int Pdim,
                     int m_per_cta, const int4* __restrict__ tiles, const int* __restrict__ tile_count,
                     int64_t out_expert_stride, uint32_t* status) {
  // Launched as a dependent of the backward GEMM (programmatic dependent
  // launch), which lets it start only once Us and Ts are complete: the next
  // gradient kernel may start at once too.
  griddep_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ps = smem;                          // kStages x 16 KiB
  uint8_t* qs = ps + kStages * kPBytes;        // kStages x 8 KiB
  Bars* bars = reinterpret_cast<Bars*>(qs + kStages * kQBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p0 = blockIdx.x * kP;
  int mbeg = blockIdx.y * m_per_cta;
  int mend = min(M, mbeg + m_per_cta);
  const bool grouped = tiles != nullptr;
  if (grouped) {
    // MoE: one token slice of one expert; its gradient is that expert's.
    if (static_cast<int>(blockIdx.y) >= *tile_count) return;
    const int4 t = tiles[blockIdx.y];
    mbeg = t.y;
    mend = min(t.z, M);
    out += t.x * out_expert_stride;
  }
  const int n_st = mend > mbeg ? (mend - mbeg + kStageM - 1) / kStageM : 0;
  volatile uint32_t* abort_word = &bars->abort_word;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->accum, 1);
    bars->abort_word = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_p);
      tma_prefetch_desc(&tm_q);
      int issued = 0;
      for (int it = 0; it < n_st; ++it) {
        const int s = it % kStages;
        if (it >= kStages &&
            !mbar_wait_short(&bars->empty[s], ((it / kStages) - 1) & 1, abort_word, status, kStatusTimeoutEmpty))
          break;
        const int m = mbeg + it * kStageM;
        mbar_arrive_expect_tx(&bars->full[s], kPBytes + kQBytes);
        tma_load_2d(ps + s * kPBytes, &tm_p, p0, m, &bars->full[s]);
        tma_load_2d(ps + s * kPBytes + kPBox, &tm_p, p0 + 64, m, &bars->full[s]);
        tma_load_2d(qs + s * kQBytes, &tm_q, 0, m, &bars->full[s]);
        ++issued;
      }
      for (int i = issued > kStages ? issued - kStages : 0; i < issued; ++i) {
        uint32_t dummy = 0;
        mbar_wait_short(&bars->full[i % kStages], (i / kStages) & 1, &dummy, status, kStatusTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // D[p, j] += P_tile^T[p, m] . Lo_tile[m, j]: A = P tile (MN-major: p
    // contiguous; two 64-p atoms 8 KiB apart), B = Lo tile (MN-major).
    const uint32_t idesc = idesc_bf16_f32_mnmn(kP, kJ);
    for (int it = 0; it < n_st; ++it) {
      const int s = it % kStages;
      if (!mbar_wait_short_warp(&bars->full[s], (it / kStages) & 1, abort_word, status, kStatusTimeoutFull)) break;
      const int valid = mend - (mbeg + it * kStageM);
      if (grouped && valid < kStageM) {
        // The tile ran into the next expert's rows: zero those rows of Lo so
        // they add nothing (a row is 128 contiguous bytes under the swizzle).
        uint4* q = reinterpret_cast<uint4*>(qs + s * kQBytes);
        for (int i = valid * 8 + lane; i < kStageM * 8; i += 32) q[i] = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
        __syncwarp();
      }
      if (lane == 0) {
        tc_fence_after();
        const uint64_t adesc = sdesc_mnmajor_sw128(smem_u32(ps + s * kPBytes), kPBox, 1024);
        const uint64_t bdesc = sdesc_mnmajor_sw128(smem_u32(qs + s * kQBytes), kQBytes, 1024);
        for (int kk = 0; kk < kStageM / 16; ++kk)
          mma_ss(tmem_base, adesc + ((2 * 1024) >> 4) * kk, bdesc + ((2 * 1024) >> 4) * kk, idesc,
                 (it | kk) != 0 ? 1u : 0u);
        tc_commit(&bars->empty[s]);
      }
      __syncwarp();
    }
    if (lane == 0) tc_commit(&bars->accum);
  } else {
    // Epilogue: lane quarter (warp & 3) holds p = p0 + 32q + lane.
    const int quarter = warp & 3;
    const int p = p0 + quarter * 32 + lane;
    // A long wait (the whole slice streams first): sleep in try_wait rather
    // than spin next to the producer and MMA warps.
    if (n_st > 0 && mbar_wait_warp(&bars->accum, 0, abort_word, status, kStatusTimeoutAccum)) {
      tc_fence_after();
      uint32_t v[2][32];
      tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16), v[0]);
      tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + 32, v[1]);
      tmem_wait_ld();
      if (p < Pdim) {
        float* row = out + p * o_sp;
        const bool vec = o_sj == 1 && (rank & 3) == 0 && (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
#pragma unroll
        for (int j = 0; j < kJ; j += 4) {
          if (j >= rank) break;
          const float a = __uint_as_float(v[j >> 5][j & 31]), b = __uint_as_float(v[j >> 5][(j & 31) + 1]);
          const float c = __uint_as_float(v[j >> 5][(j & 31) + 2]), d = __uint_as_float(v[j >> 5][(j & 31) + 3]);
          if (vec) {
            red_add_v4(row + j, a, b, c, d);
          } else {
            atomicAdd(row + j * o_sj, a);
            if (j + 1 < rank) atomicAdd(row + (j + 1) * o_sj, b);
            if (j + 2 < rank) atomicAdd(row + (j + 2) * o_sj, c);
            if (j + 3 < rank) atomicAdd(row + (j + 3) * o_sj, d);
          }
        }
      }
      tc_fence_before();
    }
  }
  // Finish no earlier than the previous launch, so completion stays ordered.
  griddep_wait();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace lg

int make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);

int launch_lora_grad(const void* P, int M, int Pdim, const void* Q, int rank, float* out, int64_t o_sp,
                     int64_t o_sj, int accumulate, cudaStream_t stream, const int4* tiles, const int* tile_count,
                     int max_tiles, int64_t out_expert_stride, int64_t out_total, bool pdl) {
  using namespace lg;
  if (Pdim % 64 != 0) return set_error(FL_ERR_ARG, "lora_grad: dim %d not a multiple of 64", Pdim);
  if (!accumulate) {
    // out is a dense [Pdim, rank] or [rank, Pdim] fp32 matrix (per expert).
    const size_t n = tiles ? static_cast<size_t>(out_total) : static_cast<size_t>(Pdim) * rank;
    cudaError_t e = cudaMemsetAsync(out, 0, n * sizeof(float), stream);
    if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "lora_grad memset: %s", cudaGetErrorString(e));
  }
  if (M < 1) return FL_OK;
  CUtensorMap tm_p, tm_q;
  int rc = make_tensor_map_2d(&tm_p, P, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, Pdim, M, static_cast<uint64_t>(Pdim) * 2,
                              64, kStageM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tensor_map_2d(&tm_q, Q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kJ, M, kJ * 2, kJ, kStageM,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms < 1)
    sms = 148;
  static bool attr_set[64] = {false};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&lora_grad_kernel),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "lora_grad attr: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  const int ptiles = (Pdim + kP - 1) / kP;
  int slices, m_per_cta;
  if (tiles) {
    slices = max_tiles;
    m_per_cta = 0;
  } else {
    // About two CTAs per SM in one wave: token slices of whole stages.
    slices = (2 * sms + ptiles - 1) / ptiles;
    const int max_slices = (M + kStageM - 1) / kStageM;
    if (slices > max_slices) slices = max_slices;
    if (slices < 1) slices = 1;
    m_per_cta = (M + slices - 1) / slices;
    m_per_cta = (m_per_cta + kStageM - 1) / kStageM * kStageM;
    slices = (M + m_per_cta - 1) / m_per_cta;
  }
  if (slices < 1) return FL_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ptiles, slices);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, lora_grad_kernel, tm_p, tm_q, out, o_sp, o_sj, rank, M, Pdim, m_per_cta,
                                     tiles, tile_count, out_expert_stride, status_word(dev));
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "lora_grad launch: %s", cudaGetErrorString(e));
  return FL_OK;
}

}  // namespace fl
