// Fused 4-bit dequantize -> tcgen05 BF16 GEMM with the LoRA branch folded into
// the same TMEM accumulation.  One kernel template serves the forward and the
// weight-gradient-free backward of the frozen projection:
//
//   forward  (kBwd = false):  Y [M,N]  = X  [M,K] . W^T    + Ts [M,r] . Blora^T
//   backward (kBwd = true) :  dX[M,K]  = dY [M,N] . W      + Us [M,r] . Alora
//
// with W[N,K] stored as the reference's group-128 record (payload uint8
// [N*K/2], two codes per byte, scales fp32 [N*K/128]), Ts = bf16(s * X.Alora^T)
// and Us = bf16(s * dY.Blora) produced by fl_lora.cu.  This replaces the
// reference's decode_into + F.linear + FP32 LoRA F.linear pair
// (ram_vram_finetune/finetune/lora.py:205-220, quantization/codecs.py:158-170)
// and its autograd backward (training/recompute.py:85-127).
//
// Mapping onto the 5th-gen tensor core ("TS" form, A operand in TMEM):
//   * MMA M (128 TMEM lanes) runs over W rows (forward) or W columns (backward);
//     MMA N (256) runs over tokens; MMA K runs over the reduction dim in 64-wide
//     stages.
//   * A = dequantized weight tile, written straight from registers into TMEM
//     by four dequant warps (tcgen05.st): the BF16 weight tile never touches
//     shared memory.
//   * B = activation tile [256 tokens x 64], TMA-loaded with the 128-byte swizzle.
//   * Packed codes arrive by TMA into a small shared-memory ring.
//   * One extra stage appends the LoRA rank (<= 64) to the K dimension: A =
//     bf16 LoRA factor rows, B = the scaled low-rank activations.
//   * D = 128 x 256 fp32 accumulator in TMEM, read back by the same four warps.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA
// issuer, warps 2-5 dequant producers then epilogue.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_codebook.cuh"
#include "fl_ptx.cuh"

namespace fl {

constexpr int kLanes = 128;         // UMMA M
constexpr int kTok = 256;           // UMMA N
constexpr int kStageK = 64;         // reduction elements per stage
constexpr int kStages = 5;
constexpr int kAccCols = 256;       // fp32 accumulator columns
constexpr int kTmemCols = 512;      // power-of-two allocation (acc + A ring)
constexpr int kAStageCols = kStageK / 2;  // bf16 pairs per lane per stage
constexpr int kXBytes = kTok * kStageK * 2;  // 32 KiB activation tile
constexpr int kQBytes = kLanes * kStageK / 2;  // 4 KiB packed-code tile
constexpr int kThreads = 192;
static_assert(kAccCols + kStages * kAStageCols <= kTmemCols, "TMEM budget");

struct GemmArgs {
  const float* scales;  // fp32 [N * K/128]
  const float* lut;     // fp32 [16]
  const float* lora;    // forward: Blora [N, r]; backward: Alora [r, K]
  __nv_bfloat16* out;   // [M, L]
  uint32_t* status;     // device status word
  int M, N, K;          // problem dims of the frozen weight W[N,K] and tokens M
  int rank;             // 0 disables the LoRA stage
};

struct __align__(8) GemmBarriers {
  uint64_t full[kStages];   // TMA bytes landed
  uint64_t afull[kStages];  // dequant warps finished writing the TMEM A stage
  uint64_t empty[kStages];  // MMAs reading the stage completed
  uint64_t accum;           // all MMAs completed
  uint32_t tmem_base;
  uint32_t abort_word;
};

constexpr int kSmemBytes = 1024 /*align slack*/ + kStages * (kXBytes + kQBytes) + sizeof(GemmBarriers);

template <bool kBwd>
__global__ void __launch_bounds__(kThreads, 1)
    fl_tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_act,   // X or dY, [M, R] bf16, box {64,256}
                      const __grid_constant__ CUtensorMap tm_low,   // Ts or Us, [M, 64] bf16, box {64,256}
                      const __grid_constant__ CUtensorMap tm_code,  // payload [N, K/2] u8
                      const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem;                                   // kStages x 32 KiB (1024-aligned)
  uint8_t* qs = smem + kStages * kXBytes;               // kStages x 4 KiB
  GemmBarriers* bars = reinterpret_cast<GemmBarriers*>(qs + kStages * kQBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = args.M, N = args.N, K = args.K;
  const int L = kBwd ? K : N;   // output columns (TMEM lane dimension)
  const int R = kBwd ? N : K;   // reduction dimension
  const int groups_per_row = K / 128;
  const int l0 = blockIdx.x * kLanes;
  const int m0 = blockIdx.y * kTok;
  const int n_main = R / kStageK;
  const bool has_lora = args.rank > 0;
  const int n_iter = n_main + (has_lora ? 1 : 0);
  volatile uint32_t* abort_word = &bars->abort_word;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->afull[s], 128);
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
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_act);
      tma_prefetch_desc(&tm_code);
      if (has_lora) tma_prefetch_desc(&tm_low);
      int issued = 0;
      for (int it = 0; it < n_iter; ++it) {
        const int s = it % kStages;
        if (it >= kStages &&
            !mbar_wait(&bars->empty[s], ((it / kStages) - 1) & 1, abort_word, args.status, kStatusTimeoutEmpty))
          break;
        if (it < n_main) {
          const int r0 = it * kStageK;
          mbar_arrive_expect_tx(&bars->full[s], kXBytes + kQBytes);
          tma_load_2d(xs + s * kXBytes, &tm_act, r0, m0, &bars->full[s]);
          if (!kBwd)
            tma_load_2d(qs + s * kQBytes, &tm_code, r0 / 2, l0, &bars->full[s]);       // 128 rows x 32 B
          else
            tma_load_2d(qs + s * kQBytes, &tm_code, l0 / 2, r0, &bars->full[s]);       // 64 rows x 64 B
        } else {
          mbar_arrive_expect_tx(&bars->full[s], kXBytes);
          tma_load_2d(xs + s * kXBytes, &tm_low, 0, m0, &bars->full[s]);
        }
        ++issued;
      }
      // Drain: never leave the CTA with bulk copies still landing in its smem.
      for (int i = issued > kStages ? issued - kStages : 0; i < issued; ++i) {
        const int s = i % kStages;
        uint32_t dummy_abort = 0;
        mbar_wait(&bars->full[s], (i / kStages) & 1, &dummy_abort, args.status, kStatusTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kLanes, kTok);
      const int lora_k_steps = (args.rank + 15) / 16;
      for (int it = 0; it < n_iter; ++it) {
        const int s = it % kStages;
        const uint32_t ph = (it / kStages) & 1;
        if (!mbar_wait(&bars->full[s], ph, abort_word, args.status, kStatusTimeoutFull)) break;
        if (!mbar_wait(&bars->afull[s], ph, abort_word, args.status, kStatusTimeoutFull)) break;
        tc_fence_after();
        const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(xs + s * kXBytes));
        const uint32_t a_col = tmem_base + kAccCols + s * kAStageCols;
        const int ksteps = it < n_main ? kStageK / 16 : lora_k_steps;
        for (int kk = 0; kk < ksteps; ++kk)
          mma_ts(tmem_base, a_col + kk * 8, bdesc + 2 * kk, idesc, (it | kk) != 0 ? 1u : 0u);
        tc_commit(&bars->empty[s]);
      }
      // Completion of every MMA issued above (also on the abort path, so TMEM
      // is never released under an in-flight MMA).
      tc_commit(&bars->accum);
      uint32_t dummy_abort = 0;
      mbar_wait(&bars->accum, 0, &dummy_abort, args.status, kStatusTimeoutAccum);
    }
  } else {
    // ------------------------------------------------ dequant producers (128 threads)
    const int quarter = warp & 3;              // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;       // lane within the 128-lane tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    float lut[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) lut[c] = __ldg(args.lut + c);
    bool ok = true;

    if (!kBwd) {
      // Thread owns weight row n; each stage decodes 64 consecutive k of it.
      const int n = l0 + row;
      const bool valid = n < N;
      const float* srow = args.scales + static_cast<size_t>(valid ? n : 0) * groups_per_row;
      float next_scale = valid ? __ldg(srow) : 0.0f;
      ProductTable table;
      for (int it = 0; it < n_iter && ok; ++it) {
        const int s = it % kStages;
        const uint32_t ph = (it / kStages) & 1;
        if (it >= kStages &&
            !mbar_wait_warp(&bars->empty[s], ((it / kStages) - 1) & 1, abort_word, args.status, kStatusTimeoutEmpty)) {
          ok = false;
          break;
        }
        uint32_t v[32];
        if (it < n_main) {
          if ((it & 1) == 0) {  // new 128-element group every two stages
            table = make_table(lut, next_scale);
            const int g_next = it / 2 + 1;
            next_scale = (valid && g_next < groups_per_row) ? __ldg(srow + g_next) : 0.0f;
          }
          if (!mbar_wait_warp(&bars->full[s], ph, abort_word, args.status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          const uint4* q = reinterpret_cast<const uint4*>(qs + s * kQBytes + row * 32);
          const uint4 q0 = q[0], q1 = q[1];
          lookup8(table, q0.x, v + 0);
          lookup8(table, q0.y, v + 4);
          lookup8(table, q0.z, v + 8);
          lookup8(table, q0.w, v + 12);
          lookup8(table, q1.x, v + 16);
          lookup8(table, q1.y, v + 20);
          lookup8(table, q1.z, v + 24);
          lookup8(table, q1.w, v + 28);
        } else {
          // LoRA stage: A row = bf16(Blora[n, 0:64]) zero padded past the rank.
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int c0 = 2 * j, c1 = 2 * j + 1;
            const float a = (valid && c0 < args.rank) ? __ldg(args.lora + static_cast<size_t>(n) * args.rank + c0) : 0.f;
            const float b = (valid && c1 < args.rank) ? __ldg(args.lora + static_cast<size_t>(n) * args.rank + c1) : 0.f;
            v[j] = pack_bf16x2(a, b);
          }
        }
        tc_fence_after();
        tmem_st_32x32b_x32(tmem_base + lane_addr + kAccCols + s * kAStageCols, v);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars->afull[s]);
      }
    } else {
      // Backward: lanes are W columns k, the stage reduces over 64 W rows n.
      // Natural-orientation bytes are decoded into 8x8 bf16 blocks in mma
      // fragment order, transposed in registers with movmatrix, and stored
      // with the 16x256b TMEM shape.  Rows are visited in the order
      // n = 16*cg + 4*(i/2) + (i%2) (+2 for odd pairs) so that after the
      // transpose each thread holds exactly the n pairs its TMEM columns need.
      const int i8 = lane >> 2;     // fragment row within an 8x8 block
      const int c4 = lane & 3;      // fragment column pair
      const int kq = quarter * 32;  // this warp's 32 k lanes inside the tile
      const int g = l0 / 128;       // all 128 lanes share one scale group
      for (int it = 0; it < n_iter && ok; ++it) {
        const int s = it % kStages;
        const uint32_t ph = (it / kStages) & 1;
        if (it >= kStages &&
            !mbar_wait_warp(&bars->empty[s], ((it / kStages) - 1) & 1, abort_word, args.status, kStatusTimeoutEmpty)) {
          ok = false;
          break;
        }
        if (it < n_main) {
          const int nbase = it * kStageK;
          float sc[8];
#pragma unroll
          for (int cg = 0; cg < 4; ++cg) {
#pragma unroll
            for (int odd = 0; odd < 2; ++odd) {
              const int nr = 16 * cg + 4 * (i8 >> 1) + (i8 & 1) + 2 * odd;
              sc[cg * 2 + odd] = __ldg(args.scales + static_cast<size_t>(nbase + nr) * groups_per_row + g);
            }
          }
          if (!mbar_wait_warp(&bars->full[s], ph, abort_word, args.status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int cg = 0; cg < 4; ++cg) {
            uint32_t frag[2][4];  // [odd][byte slot]
#pragma unroll
            for (int odd = 0; odd < 2; ++odd) {
              const int nr = 16 * cg + 4 * (i8 >> 1) + (i8 & 1) + 2 * odd;
              const uint4 seg = *reinterpret_cast<const uint4*>(qs + s * kQBytes + nr * 64 + kq / 2);
              // bytes c4, 4+c4, 8+c4, 12+c4 of the 16-byte segment
              const uint32_t sel = static_cast<uint32_t>(c4) | (static_cast<uint32_t>(c4 + 4) << 4);
              const uint32_t b01 = prmt(seg.x, seg.y, sel);
              const uint32_t b23 = prmt(seg.z, seg.w, sel);
              const uint32_t bytes = prmt(b01, b23, 0x5410);
              const float scale = sc[cg * 2 + odd];
#pragma unroll
              for (int b = 0; b < 4; ++b) {
                const uint32_t byte = (bytes >> (8 * b)) & 0xFFu;
                const float lo = __fmul_rn(lut[byte & 15u], scale);
                const float hi = __fmul_rn(lut[byte >> 4], scale);
                frag[odd][b] = pack_bf16x2(lo, hi);
              }
            }
            // byte slot b: (h = b/2, +8 k columns when b odd)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t r0 = movmatrix_trans(frag[0][2 * h + 0]);
              const uint32_t r1 = movmatrix_trans(frag[1][2 * h + 0]);
              const uint32_t r2 = movmatrix_trans(frag[0][2 * h + 1]);
              const uint32_t r3 = movmatrix_trans(frag[1][2 * h + 1]);
              const uint32_t taddr = tmem_base + (static_cast<uint32_t>(kq + 16 * h) << 16) + kAccCols +
                                     s * kAStageCols + cg * 8;
              tmem_st_16x256b_x1(taddr, r0, r1, r2, r3);
            }
          }
        } else {
          // LoRA stage: lane k holds bf16(Alora[0:64, k]) zero padded past the rank.
          const int k = l0 + row;
          uint32_t v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int c0 = 2 * j, c1 = 2 * j + 1;
            const float a = c0 < args.rank ? __ldg(args.lora + static_cast<size_t>(c0) * K + k) : 0.f;
            const float b = c1 < args.rank ? __ldg(args.lora + static_cast<size_t>(c1) * K + k) : 0.f;
            v[j] = pack_bf16x2(a, b);
          }
          tc_fence_after();
          tmem_st_32x32b_x32(tmem_base + lane_addr + kAccCols + s * kAStageCols, v);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars->afull[s]);
      }
    }

    // ------------------------------------------------------------ epilogue
    if (ok && mbar_wait_warp(&bars->accum, 0, abort_word, args.status, kStatusTimeoutAccum)) {
      tc_fence_after();
      const int l = l0 + row;
      const bool lvalid = l < L;
#pragma unroll 1
      for (int c = 0; c < kTok / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + lane_addr + c * 32, v);
        tmem_wait_ld();
        if (lvalid) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = m0 + c * 32 + j;
            if (m < M) args.out[static_cast<size_t>(m) * L + l] = __float2bfloat16_rn(__uint_as_float(v[j]));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace fl

// ------------------------------------------------------------------ host side
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "fl_host.h"

namespace fl {

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

static int make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes,
                       uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                       uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = get_encode_fn();
  if (!fn) return set_error(FL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return FL_OK;
}

static int ensure_smem_attr(const void* kernel) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  return FL_OK;
}

// act: [M, R] bf16 activations; low: [M, 64] bf16 low-rank activations (may be
// null when rank == 0); codes/scales: the frozen record; out: [M, L] bf16.
int launch_tc_gemm(bool bwd, const void* act, const void* low, const uint8_t* codes, const float* scales,
                   const float* lut, const float* lora, int rank, void* out, int M, int N, int K,
                   uint32_t* status, cudaStream_t stream) {
  const int L = bwd ? K : N, R = bwd ? N : K;
  CUtensorMap tm_act, tm_low, tm_code;
  int rc = make_map_2d(&tm_act, act, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, R, M, static_cast<uint64_t>(R) * 2, 64,
                       256, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (rank > 0) {
    rc = make_map_2d(&tm_low, low, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64, M, 128, 64, 256,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    tm_low = tm_act;
  }
  if (!bwd)
    rc = make_map_2d(&tm_code, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, K / 2, 32, 128,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
  else
    rc = make_map_2d(&tm_code, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, K / 2, 64, 64,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  GemmArgs a;
  a.scales = scales;
  a.lut = lut;
  a.lora = lora;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.status = status;
  a.M = M;
  a.N = N;
  a.K = K;
  a.rank = rank;
  dim3 grid((L + kLanes - 1) / kLanes, (M + kTok - 1) / kTok);
  if (!bwd) {
    static bool attr = false;
    if (!attr) { if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(&fl_tc_gemm_kernel<false>)))) return rc; attr = true; }
    fl_tc_gemm_kernel<false><<<grid, kThreads, kSmemBytes, stream>>>(tm_act, tm_low, tm_code, a);
  } else {
    static bool attr = false;
    if (!attr) { if ((rc = ensure_smem_attr(reinterpret_cast<const void*>(&fl_tc_gemm_kernel<true>)))) return rc; attr = true; }
    fl_tc_gemm_kernel<true><<<grid, kThreads, kSmemBytes, stream>>>(tm_act, tm_low, tm_code, a);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "tc_gemm launch: %s", cudaGetErrorString(e));
  return FL_OK;
}

}  // namespace fl
