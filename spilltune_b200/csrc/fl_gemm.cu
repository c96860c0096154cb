// Fused 4-bit dequantize -> tcgen05 BF16 GEMM with the LoRA branch folded into
// the same TMEM accumulation, forward of the frozen projection:
//
//   Y [M,N] = X [M,K] . W^T + Ts [M,r] . Blora^T
//
// (the backward lives in fl_gemm_bwd.cu)
// with W[N,K] stored as the reference's group-128 record (payload uint8
// [N*K/2], two codes per byte, scales fp32 [N*K/128]), Ts = bf16(s * X.Alora^T)
// produced by fl_lora.cu.  This replaces the reference's decode_into + F.linear +
// FP32 LoRA F.linear pair (ram_vram_finetune/finetune/lora.py:205-220,
// quantization/codecs.py:158-170).
//
// Mapping onto the 5th-gen tensor core ("TS" form, A operand in TMEM), run by
// a CTA pair (cluster of 2, tcgen05 cta_group::2):
//   * MMA M (256 = 128 TMEM lanes in each CTA) runs over W rows; MMA N (256)
//     runs over tokens, each CTA holding the
//     shared-memory half of its 128 tokens; MMA K runs over the reduction dim
//     in 64-wide stages.  The pair halves the activation bytes each SM loads
//     and stores per FLOP compared with one CTA.
//   * A = dequantized weight tile, written straight from registers into TMEM
//     by four dequant warps (tcgen05.st): the BF16 weight tile never touches
//     shared memory.
//   * B = activation tile [128 tokens x 64] per CTA, TMA-loaded (no multicast)
//     with the 128-byte swizzle.
//   * Packed codes arrive by TMA into a small shared-memory ring.
//   * One extra stage appends the LoRA rank (<= 64) to the K dimension: A =
//     bf16(Blora) rows, B = the scaled low-rank activations Ts.
//   * D = 256 x 256 fp32 accumulator, 128 rows in each CTA's TMEM, read back by
//     the dequant warps of that CTA.
//
// Warp roles (448 threads per CTA): warp 0 TMA producer, warp 1 TMEM owner
// (both CTAs) + MMA issuer (leader CTA only), warps 2-13 dequant producers in
// three groups of four that take turns on pairs of stages (one warp per TMEM
// lane quarter decodes the whole stage for its lanes), then epilogue.
// Synchronisation: full[s] (local TMA bytes), afull[s] (leader only: 8 local +
// 8 peer dequant-warp arrivals), empty[s] and accum (multicast tcgen05.commit
// from the leader into both CTAs).
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_codebook.cuh"
#include "fl_ptx.cuh"

namespace fl {

constexpr int kLanes = 128;         // W rows (or columns) per CTA; UMMA M = 256 per pair
constexpr int kTok = 256;           // UMMA N (tokens per pair tile)
constexpr int kTokHalf = 128;       // tokens whose activations each CTA holds
constexpr int kStageK = 64;         // reduction elements per stage
constexpr int kStages = 8;
constexpr int kGroupM = 8;          // token tiles per band of the grouped tile order
constexpr int kAccCols = 256;       // fp32 accumulator columns
constexpr int kTmemCols = 512;      // power-of-two allocation (acc + A ring)
constexpr int kAStageCols = kStageK / 2;  // bf16 pairs per lane per stage
constexpr int kXBytes = kTokHalf * kStageK * 2;  // 16 KiB activation half-tile
constexpr int kQBytes = kLanes * kStageK / 2;  // 4 KiB packed-code tile
constexpr int kGroups = 3;                     // dequant warp groups (4 warps each)
constexpr int kThreads = 64 + 128 * kGroups;   // 2 control warps + dequant/epilogue warps
static_assert(kAccCols + kStages * kAStageCols <= kTmemCols, "TMEM budget");

struct GemmArgs {
  const float* scales;  // fp32 [N * K/128]
  const float* lut;     // fp32 [16]
  const float* lora;    // forward: Blora [N, r]; backward: Alora [r, K]
  __nv_bfloat16* out;   // [M, L]
  uint32_t* status;     // device status word
  int M, N, K;          // problem dims of the frozen weight W[N,K] and tokens M
  int rank;             // 0 disables the LoRA stage
  // Grouped (MoE) launches: tile list {expert, first row, end row, weight tile}
  // over expert-sorted token rows, its length on the device; null for one weight.
  const int4* tiles;
  const int* tile_count;
};

struct __align__(16) GemmBarriers {
  uint64_t full[kStages];   // TMA bytes landed
  uint64_t afull[kStages];  // leader: both CTAs' dequant warps finished the TMEM A stage
  uint64_t empty[kStages];  // MMAs reading the stage completed
  uint64_t accum;           // all MMAs completed
  uint32_t tmem_base;
  uint32_t abort_word;
  alignas(16) float lut[16];  // codebook copy for the decoders
};

constexpr int kSmemBytes = 1024 /*align slack*/ + kStages * (kXBytes + kQBytes) + sizeof(GemmBarriers);

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
  const int L = N;   // output columns (TMEM lane dimension)
  const int R = K;   // reduction dimension
  const int groups_per_row = K / 128;
  const uint32_t crank = cluster_ctarank();       // 0 = leader of the CTA pair
  int w_tile, m_tile;
  int expert = 0, m_end = M;
  int m0;                                           // first token of the pair tile
  if (args.tiles != nullptr) {
    // MoE: one tile of <= 256 rows of one expert's token segment.  Both CTAs
    // of the pair read the same entry, so they leave together.
    const int pair = blockIdx.x >> 1;
    if (pair >= *args.tile_count) return;
    const int4 t = args.tiles[pair];
    expert = t.x;
    m0 = t.y;
    m_end = t.z;
    w_tile = t.w;
    m_tile = 0;
  } else {
    // Grouped tile order: pairs that run at the same time cover a band of
    // kGroupM token tiles x several weight tiles, so an activation tile is
    // requested by a handful of pairs at once instead of by every SM.
    const int num_w = (L + 2 * kLanes - 1) / (2 * kLanes);
    const int num_m = (M + kTok - 1) / kTok;
    const int pair = blockIdx.x >> 1;
    const int band = pair / (kGroupM * num_w);
    const int first_m = band * kGroupM;
    const int rows_in_band = min(kGroupM, num_m - first_m);
    const int local = pair - band * kGroupM * num_w;
    m_tile = first_m + local % rows_in_band;
    w_tile = local / rows_in_band;
    m0 = m_tile * kTok;
  }
  const int l0 = w_tile * (2 * kLanes) + static_cast<int>(crank) * kLanes;
  const int wrow0 = expert * N;                     // this expert's first row in the stacked record
  const int mh = m0 + static_cast<int>(crank) * kTokHalf;  // first token of this CTA's half
  const int n_main = R / kStageK;
  const bool has_lora = args.rank > 0;
  const int n_iter = n_main + (has_lora ? 1 : 0);
  volatile uint32_t* abort_word = &bars->abort_word;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->afull[s], 2 * 4);  // one arrival per dequant warp of the owning group, both CTAs
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->accum, 1);
    bars->abort_word = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < 16) {
    bars->lut[threadIdx.x] = __ldg(args.lut + threadIdx.x);
  }
  if (warp == 1) {
    tmem_alloc2(&bars->tmem_base, kTmemCols);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // peer barriers initialised before any remote arrive
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
          tma_load_2d(xs + s * kXBytes, &tm_act, r0, mh, &bars->full[s]);
          tma_load_2d(qs + s * kQBytes, &tm_code, r0 / 2, wrow0 + l0, &bars->full[s]);  // 128 rows x 32 B
        } else {
          mbar_arrive_expect_tx(&bars->full[s], kXBytes);
          tma_load_2d(xs + s * kXBytes, &tm_low, 0, mh, &bars->full[s]);
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
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (lane == 0 && crank == 0) {
      const uint32_t idesc = idesc_bf16_f32(2 * kLanes, kTok);
      const int lora_k_steps = (args.rank + 15) / 16;
      for (int it = 0; it < n_iter; ++it) {
        const int s = it % kStages;
        const uint32_t ph = (it / kStages) & 1;
        // Every dequant warp of both CTAs arrives only after its own CTA's
        // TMA bytes for the stage landed, so afull covers both B halves too.
        if (!mbar_wait_cluster(&bars->afull[s], ph, abort_word, args.status, kStatusTimeoutFull)) break;
        tc_fence_after();
        const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(xs + s * kXBytes));
        const uint32_t a_col = tmem_base + kAccCols + s * kAStageCols;
        const int ksteps = it < n_main ? kStageK / 16 : lora_k_steps;
        for (int kk = 0; kk < ksteps; ++kk)
          mma_ts2(tmem_base, a_col + kk * 8, bdesc + 2 * kk, idesc, (it | kk) != 0 ? 1u : 0u);
        tc_commit2_mc(&bars->empty[s], 0x3);
      }
      // Completion of every MMA issued above (also on the abort path, so TMEM
      // is never released under an in-flight MMA).
      tc_commit2_mc(&bars->accum, 0x3);
      uint32_t dummy_abort = 0;
      mbar_wait(&bars->accum, 0, &dummy_abort, args.status, kStatusTimeoutAccum);
    }
  } else {
    // ----------------------------------- dequant producers (kGroups x 4 warps)
    // Within a group: one warp per TMEM lane quarter decodes the whole stage
    // for its 32 lanes.  Groups take turns on pairs of stages (one 128-wide
    // scale group), so each warp has kGroups pair-times to hide its barrier,
    // shared-memory and TMEM-store latencies.
    const int dw = warp - 2;                   // dequant warp index
    const int grp = dw >> 2;                   // stage-pair group of this warp
    const int quarter = warp & 3;              // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;       // lane within the 128-lane tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t afull_leader = mapa_shared(smem_u32(&bars->afull[0]), 0);
    const float* lut_s = bars->lut;
    bool ok = true;

    {
      // Thread owns weight row n; each stage it decodes the 64 k of the stage
      // (32 TMEM columns).
      const int n = l0 + row;
      const bool valid = n < N;
      const float* srow = args.scales + static_cast<size_t>(wrow0 + (valid ? n : 0)) * groups_per_row;
      float next_scale = (valid && 2 * grp < 2 * groups_per_row) ? __ldg(srow + grp) : 0.0f;
      for (int pit = 2 * grp; pit < n_iter && ok; pit += 2 * kGroups) {
        ProductTable table;
        if (pit < n_main) {
          table = make_table(lut_s, next_scale);
          const int g_next = pit / 2 + kGroups;
          next_scale = (valid && g_next < groups_per_row) ? __ldg(srow + g_next) : 0.0f;
        }
        for (int it = pit; it < pit + 2 && it < n_iter; ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (it >= kStages &&
              !mbar_wait_warp(&bars->empty[s], ((it / kStages) - 1) & 1, abort_word, args.status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (!mbar_wait_warp(&bars->full[s], ph, abort_word, args.status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          uint32_t v[32];
          if (it < n_main) {
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
              const int c0 = 2 * j, c1 = c0 + 1;
              const float a = (valid && c0 < args.rank) ? __ldg(args.lora + static_cast<size_t>(wrow0 + n) * args.rank + c0) : 0.f;
              const float b = (valid && c1 < args.rank) ? __ldg(args.lora + static_cast<size_t>(wrow0 + n) * args.rank + c1) : 0.f;
              v[j] = pack_bf16x2(a, b);
            }
          }
          tc_fence_after();
          tmem_st_32x32b_x32(tmem_base + lane_addr + kAccCols + s * kAStageCols, v);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(afull_leader + s * 8);
        }
      }
    }
    // A group that stopped early (abort) must not leave others waiting forever:
    // the bounded waits and the abort word end them.
    ok = __all_sync(0xffffffffu, ok) != 0;

    // ------------------------------------------------------------ epilogue
    // The kGroups warps of each lane quarter take the 32-column token chunks
    // round robin.
    if (ok && mbar_wait_warp(&bars->accum, 0, abort_word, args.status, kStatusTimeoutAccum)) {
      tc_fence_after();
      const int l = l0 + row;
      const bool lvalid = l < L;
#pragma unroll 1
      for (int c = 32 * grp; c < kTok; c += 32 * kGroups) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + lane_addr + c, v);
        tmem_wait_ld();
        if (lvalid) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = m0 + c + j;
            if (m < m_end) args.out[static_cast<size_t>(m) * L + l] = __float2bfloat16_rn(__uint_as_float(v[j]));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs done with TMEM and with each other's barriers
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc2(tmem_base, kTmemCols);
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

int make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = get_encode_fn();
  if (!fn) return set_error(FL_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  // The encode is a driver call: make the runtime's current device's primary
  // context current on this thread first (e.g. torch's autograd worker thread
  // may not have touched the runtime yet).
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess)
    return set_error(FL_ERR_CUDA, "no current CUDA device for the tensor map");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return FL_OK;
}

// x: [M, K] bf16 activations; ts: [M, 64] bf16 scaled low-rank activations
// (unused when rank == 0); codes/scales/lut: the frozen record W[N, K];
// blora: [N, rank] fp32; y: [M, N] bf16.
int launch_fwd_gemm(const void* x, const void* ts, const uint8_t* codes, const float* scales, const float* lut,
                    const float* blora, int rank, void* y, int M, int N, int K, uint32_t* status,
                    cudaStream_t stream, const int4* tiles, const int* tile_count, int experts, int max_tiles) {
  CUtensorMap tm_act, tm_low, tm_code;
  int rc = make_tensor_map_2d(&tm_act, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, K, M, static_cast<uint64_t>(K) * 2, 64,
                              kTokHalf, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (rank > 0) {
    rc = make_tensor_map_2d(&tm_low, ts, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 64, M, 128, 64, kTokHalf,
                            CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    tm_low = tm_act;
  }
  rc = make_tensor_map_2d(&tm_code, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, static_cast<uint64_t>(N) * experts,
                          K / 2, 32, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  GemmArgs a;
  a.scales = scales;
  a.lut = lut;
  a.lora = blora;
  a.out = static_cast<__nv_bfloat16*>(y);
  a.status = status;
  a.M = M;
  a.N = N;
  a.K = K;
  a.rank = rank;
  a.tiles = tiles;
  a.tile_count = tile_count;
  // CTA pairs: each pair covers 256 W rows x 256 tokens (grouped: one listed tile).
  dim3 grid(tiles ? 2 * max_tiles : 2 * ((N + 2 * kLanes - 1) / (2 * kLanes)) * ((M + kTok - 1) / kTok));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&fl_tc_gemm_kernel),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  cudaError_t le = cudaLaunchKernelEx(&cfg, fl_tc_gemm_kernel, tm_act, tm_low, tm_code, a);
  if (le != cudaSuccess) return set_error(FL_ERR_CUDA, "fwd gemm launch: %s", cudaGetErrorString(le));
  return FL_OK;
}

}  // namespace fl
