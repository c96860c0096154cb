// lora_down: the low-rank projection of the LoRA branch,
//
//   Lo[m, j] = bf16( s * sum_r P[m, r] * Q(j, r) ),  j < rank (<= 64), zero for rank <= j < 64,
//
// forward: P = X, Q = Alora (the reference's F.linear(x.float(), A),
// finetune/lora.py:219) -> Ts;  backward: P = dY, Q = Blora^T (the VJP factor
// dY.float() @ B, training/recompute.py:102-105) -> Us.
//
// HBM-bound: it streams P once.  Each CTA owns 128 rows of P and one slice of
// the reduction dimension; the 4 CTAs of a cluster split the reduction and
// add their partial sums through distributed shared memory, so no workspace
// is needed.  P tiles arrive by TMA (128-byte swizzle); two warps turn the
// matching chunk of the FP32 factor into a bf16 hi/lo pair (~16 mantissa bits)
// in the same swizzled K-major layout; one thread issues tcgen05 MMAs
// (M = 128 rows, N = padded rank, K = 64 per stage) into a TMEM accumulator.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {
namespace ld {

constexpr int kRows = 128;
constexpr int kStageR = 64;
constexpr int kSplit = 4;                       // CTAs per cluster along the reduction
constexpr int kThreads = 128;
constexpr int kPBytes = kRows * kStageR * 2;    // 16 KiB

template <int NQ>
struct Cfg {
  static constexpr int kStages = NQ == 64 ? 6 : 4;
  static constexpr int kQBytes = NQ * kStageR * 2;        // one bf16 plane of the factor chunk
  static constexpr int kTmemCols = NQ < 32 ? 32 : NQ;
  static constexpr int kRedBytes = (kSplit - 1) * kRows * NQ * 4;  // peers' partials (reuses P stages)
  static_assert(kRedBytes <= kStages * kPBytes, "partial buffer must fit in the P stages");
  static constexpr int kSmemBytes = 1024 + kStages * (kPBytes + 2 * kQBytes) + 256;
};

struct __align__(8) Bars {
  uint64_t pfull[6];
  uint64_t qfull[6];
  uint64_t empty[6];
  uint64_t accum;
  uint32_t tmem_base;
  uint32_t abort_word;
};

template <int NQ>
__global__ void __launch_bounds__(kThreads, 1)
    lora_down_tc_kernel(const __grid_constant__ CUtensorMap tm_p, const float* __restrict__ q, int64_t q_sj,
                        int64_t q_sr, int rank, float s, __nv_bfloat16* __restrict__ out, int M, int R,
                        uint32_t* status, const int4* tiles, const int* tile_count, int64_t q_expert_stride) {
  using C = Cfg<NQ>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ps = smem;                                    // kStages x 16 KiB
  uint8_t* qh = ps + C::kStages * kPBytes;               // kStages x kQBytes (hi)
  uint8_t* ql = qh + C::kStages * C::kQBytes;            // kStages x kQBytes (lo)
  Bars* bars = reinterpret_cast<Bars*>(ql + C::kStages * C::kQBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  int m0 = (blockIdx.x / kSplit) * kRows;
  int m_end = M;
  if (tiles != nullptr) {
    // MoE: one <= 128-row tile of one expert's segment; its factor is that
    // expert's.  The 4 CTAs of the cluster read the same entry.
    const int ti = blockIdx.x / kSplit;
    if (ti >= *tile_count) return;
    const int4 t = tiles[ti];
    m0 = t.y;
    m_end = t.z;
    q += t.x * q_expert_stride;
  }
  const int n_chunks = R / kStageR;
  const int c_begin = static_cast<int>(crank) * n_chunks / kSplit;
  const int c_end = (static_cast<int>(crank) + 1) * n_chunks / kSplit;
  const int n_iter = c_end - c_begin;
  volatile uint32_t* abort_word = &bars->abort_word;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&bars->pfull[i], 1);
      mbar_init(&bars->qfull[i], 2);
      mbar_init(&bars->empty[i], 1);
    }
    mbar_init(&bars->accum, 1);
    bars->abort_word = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_p);
      int issued = 0;
      for (int it = 0; it < n_iter; ++it) {
        const int st = it % C::kStages;
        if (it >= C::kStages &&
            !mbar_wait_short(&bars->empty[st], ((it / C::kStages) - 1) & 1, abort_word, status, kStatusTimeoutEmpty))
          break;
        mbar_arrive_expect_tx(&bars->pfull[st], kPBytes);
        tma_load_2d(ps + st * kPBytes, &tm_p, (c_begin + it) * kStageR, m0, &bars->pfull[st]);
        ++issued;
      }
      for (int i = issued > C::kStages ? issued - C::kStages : 0; i < issued; ++i) {
        uint32_t dummy = 0;
        mbar_wait_short(&bars->pfull[i % C::kStages], (i / C::kStages) & 1, &dummy, status, kStatusTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kRows, NQ);
      for (int it = 0; it < n_iter; ++it) {
        const int st = it % C::kStages;
        const uint32_t ph = (it / C::kStages) & 1;
        if (!mbar_wait_short(&bars->pfull[st], ph, abort_word, status, kStatusTimeoutFull)) break;
        if (!mbar_wait_short(&bars->qfull[st], ph, abort_word, status, kStatusTimeoutFull)) break;
        tc_fence_after();
        const uint64_t pd = sdesc_kmajor_sw128(smem_u32(ps + st * kPBytes));
        const uint64_t hd = sdesc_kmajor_sw128(smem_u32(qh + st * C::kQBytes));
        const uint64_t lo = sdesc_kmajor_sw128(smem_u32(ql + st * C::kQBytes));
        for (int kk = 0; kk < kStageR / 16; ++kk) {
          mma_ss(tmem_base, pd + 2 * kk, hd + 2 * kk, idesc, (it | kk) != 0 ? 1u : 0u);
          mma_ss(tmem_base, pd + 2 * kk, lo + 2 * kk, idesc, 1u);
        }
        tc_commit(&bars->empty[st]);
      }
      tc_commit(&bars->accum);
      uint32_t dummy = 0;
      mbar_wait_short(&bars->accum, 0, &dummy, status, kStatusTimeoutAccum);
    }
  } else {
    // Factor converters: chunk (j, 8 consecutive r) -> 16-byte hi and lo pieces
    // at row j, chunk position c ^ (j % 8) of the 128-byte-swizzled tile.  The
    // FP32 chunks of the next kAhead stages are loaded into registers before the
    // current one is converted, so the global-load latency overlaps.
    constexpr int kPer = NQ / 8;                 // chunks per thread per stage (NQ*8 chunks, 64 threads)
    constexpr int kAhead = NQ <= 32 ? 2 : 1;
    const int t = threadIdx.x - 64;
    float buf[kAhead + 1][kPer][8];
    auto fetch = [&](int it, float (&v)[kPer][8]) {
      const int r0 = (c_begin + it) * kStageR;
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int idx = t + 64 * u;
        const int j = idx >> 3, c = idx & 7;
        if (it < n_iter && j < rank) {
          const float* src = q + j * q_sj + static_cast<int64_t>(r0 + 8 * c) * q_sr;
          if (q_sr == 1) {
            const float4 a = __ldg(reinterpret_cast<const float4*>(src));
            const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
            v[u][0] = a.x; v[u][1] = a.y; v[u][2] = a.z; v[u][3] = a.w;
            v[u][4] = b.x; v[u][5] = b.y; v[u][6] = b.z; v[u][7] = b.w;
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[u][e] = __ldg(src + e * q_sr);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) v[u][e] = 0.f;
        }
      }
    };
#pragma unroll
    for (int a = 0; a < kAhead; ++a) fetch(a, buf[a]);
    for (int it = 0; it < n_iter && ok; ++it) {
      const int st = it % C::kStages;
      fetch(it + kAhead, buf[kAhead]);
      if (it >= C::kStages &&
          !mbar_wait_short_warp(&bars->empty[st], ((it / C::kStages) - 1) & 1, abort_word, status, kStatusTimeoutEmpty)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int idx = t + 64 * u;
        const int j = idx >> 3, c = idx & 7;
        uint32_t h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          h[e] = pack_bf16x2(buf[0][u][2 * e], buf[0][u][2 * e + 1]);
          const float h0 = __uint_as_float(h[e] << 16), h1 = __uint_as_float(h[e] & 0xFFFF0000u);
          l[e] = pack_bf16x2(buf[0][u][2 * e] - h0, buf[0][u][2 * e + 1] - h1);
        }
        const uint32_t off = j * 128 + ((c ^ (j & 7)) << 4);
        *reinterpret_cast<uint4*>(qh + st * C::kQBytes + off) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(ql + st * C::kQBytes + off) = make_uint4(l[0], l[1], l[2], l[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->qfull[st]);
#pragma unroll
      for (int a = 0; a < kAhead; ++a)
#pragma unroll
        for (int u = 0; u < kPer; ++u)
#pragma unroll
          for (int e = 0; e < 8; ++e) buf[a][u][e] = buf[a + 1][u][e];
    }
  }

  // ---------------------------------------------------------------- reduction
  // All 4 warps: lane quarter w holds rows 32w..32w+31 of the CTA's 128.
  const int row = warp * 32 + lane;
  float acc[NQ];
  bool have = false;
  if (n_iter > 0 && mbar_wait_short_warp(&bars->accum, 0, abort_word, status, kStatusTimeoutAccum)) {
    tc_fence_after();
#pragma unroll
    for (int c0 = 0; c0 < NQ; c0 += 16) {
      uint32_t v[16];
      tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(warp * 32) << 16) + c0, v);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[c0 + e] = __uint_as_float(v[e]);
    }
    have = true;
  }
  if (!have) {
#pragma unroll
    for (int e = 0; e < NQ; ++e) acc[e] = 0.f;
  }
  // Round 1: every CTA finished its main loop, so rank 0's stage buffers are free.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  float* red = reinterpret_cast<float*>(ps);  // [kSplit-1][kRows][NQ] in rank 0
  if (crank != 0) {
    const uint32_t base = mapa_shared(smem_u32(red), 0) +
                          static_cast<uint32_t>(((crank - 1) * kRows + row) * NQ * 4);
#pragma unroll
    for (int e = 0; e < NQ; ++e) st_shared_cluster_u32(base + 4 * e, __float_as_uint(acc[e]));
  }
  cluster_sync();
  if (crank == 0) {
#pragma unroll 1
    for (int p = 0; p < kSplit - 1; ++p) {
      const float* pr = red + (p * kRows + row) * NQ;
#pragma unroll
      for (int e = 0; e < NQ; ++e) acc[e] += pr[e];
    }
    const int m = m0 + row;
    if (m < m_end) {
      uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(m) * 64);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j0 = 8 * c + 2 * e, j1 = j0 + 1;
          const float a = (j0 < NQ && j0 < rank) ? s * acc[j0 < NQ ? j0 : 0] : 0.f;
          const float b = (j1 < NQ && j1 < rank) ? s * acc[j1 < NQ ? j1 : 0] : 0.f;
          w[e] = pack_bf16x2(a, b);
        }
        dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

template <int NQ>
static int launch_nq(const CUtensorMap& tm, const float* q, int64_t q_sj, int64_t q_sr, int rank, float s,
                     void* out, int M, int R, cudaStream_t stream, const int4* tiles, const int* tile_count,
                     int max_tiles, int64_t q_expert_stride) {
  using C = Cfg<NQ>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&lora_down_tc_kernel<NQ>),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "lora_down attr: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  uint32_t* status = status_word(dev);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kSplit * (tiles ? max_tiles : (M + kRows - 1) / kRows));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t le = cudaLaunchKernelEx(&cfg, lora_down_tc_kernel<NQ>, tm, q, q_sj, q_sr, rank, s,
                                      static_cast<__nv_bfloat16*>(out), M, R, status, tiles, tile_count,
                                      q_expert_stride);
  if (le != cudaSuccess) return set_error(FL_ERR_CUDA, "lora_down launch: %s", cudaGetErrorString(le));
  return FL_OK;
}

}  // namespace ld

int make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);

int launch_lora_down(const void* P, int M, int R, const float* q, int64_t q_sj, int64_t q_sr, int rank, float s,
                     void* out64, cudaStream_t stream, const int4* tiles, const int* tile_count, int max_tiles,
                     int64_t q_expert_stride) {
  if (R % 128 != 0) return set_error(FL_ERR_ARG, "lora_down: reduction dim %d not a multiple of 128", R);
  if (rank < 1 || rank > 64) return set_error(FL_ERR_ARG, "lora_down: rank %d outside [1, 64]", rank);
  if (q_sr == 1 && (reinterpret_cast<uintptr_t>(q) & 15u))
    return set_error(FL_ERR_ARG, "lora_down: factor must be 16-byte aligned");
  CUtensorMap tm;
  int rc = make_tensor_map_2d(&tm, P, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, R, M, static_cast<uint64_t>(R) * 2, 64,
                              ld::kRows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (rank <= 16)
    return ld::launch_nq<16>(tm, q, q_sj, q_sr, rank, s, out64, M, R, stream, tiles, tile_count, max_tiles,
                             q_expert_stride);
  if (rank <= 32)
    return ld::launch_nq<32>(tm, q, q_sj, q_sr, rank, s, out64, M, R, stream, tiles, tile_count, max_tiles,
                             q_expert_stride);
  return ld::launch_nq<64>(tm, q, q_sj, q_sr, rank, s, out64, M, R, stream, tiles, tile_count, max_tiles,
                           q_expert_stride);
}

}  // namespace fl
