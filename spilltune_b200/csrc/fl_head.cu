// Chunked LM head + shifted cross-entropy (the reference's terminal:
// ram_vram_finetune/quantization/native_terminal.py:11-47, _ChunkedCE, and the
// same loop in training/engine.py:58-78).  Per token chunk the reference runs
//   logits = F.linear(h, head)                          (bf16, [T, V])
//   ce     = cross_entropy(logits.float(), target, ignore_index=-100, sum)
//   dh     = autograd of ce / normalization             (bf16, [T, H])
// Here the chunk is four launches:
//   1. logits GEMM (h . head^T) whose epilogue rounds each accumulator tile to
//      bf16, stores it, and reduces the ROUNDED values of its 256 vocabulary
//      columns to a per-row (max, sum exp) partial and, where the row's
//      target falls in the tile, the target logit;
//   2. a row kernel: log-sum-exp over the partials, the summed loss;
//   3. dlogits = (softmax - onehot) / normalization, rounded to bf16, in place;
//   4. dh GEMM (dlogits . head, the head entering MN-major).
// Both GEMMs are one persistent CTA-pair tcgen05 kernel with TMA for both
// operands and two TMEM accumulators (the next tile accumulates while the
// previous one drains).  The head is frozen: no head gradient.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {

int make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);

namespace hd {

constexpr int kHalf = 128;                  // A rows (tokens) and B rows (N) per CTA
constexpr int kStageK = 64;
constexpr int kStages = 6;
constexpr int kGroupM = 8;                  // token tiles per band of the tile order
constexpr int kEpiWarps = 4;                // one per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kAccCols = 256;
constexpr int kTmemCols = 2 * kAccCols;
constexpr int kABytes = kHalf * kStageK * 2;  // 16 KiB
constexpr int kBBytes = kHalf * kStageK * 2;  // 16 KiB
constexpr int kIgnore = -100;

enum Epi { kEpiStore = 0, kEpiCE = 1 };

struct __align__(16) Bars {
  uint64_t full[kStages];      // local TMA bytes of the stage
  uint64_t pfull[kStages];     // leader: the peer's TMA bytes landed (relayed)
  uint64_t empty[kStages];     // MMAs reading the stage completed (multicast commit)
  uint64_t accum[2];
  uint64_t acc_empty[2];       // leader: both CTAs' epilogue warps drained accumulator b
  uint32_t tmem_base;
  uint32_t abort_word;
};

constexpr int kSmemBytes = 1024 + kStages * (kABytes + kBBytes) + static_cast<int>(sizeof(Bars));

struct Args {
  __nv_bfloat16* out;      // [M, N] bf16, row stride ldo
  int64_t ldo;
  uint32_t* status;
  int M, N, K;
  // kEpiCE: targets of the rows (kIgnore = none), partials [M, n_tiles] (max, sum),
  // target logits [M].
  const int64_t* targets;
  float2* part;
  float* tgt;
};

struct Tile {
  int m0, n0;
};
__device__ __forceinline__ Tile tile_at(int t, int num_m, int num_n) {
  const int band = t / (kGroupM * num_n);
  const int first_m = band * kGroupM;
  const int rows_in_band = min(kGroupM, num_m - first_m);
  const int local = t - band * kGroupM * num_n;
  Tile r;
  r.m0 = (first_m + local % rows_in_band) * 2 * kHalf;
  r.n0 = (local / rows_in_band) * 2 * kHalf;
  return r;
}

// D[m, n] = sum_k A[m, k] B(k, n): A [M, K] K-major; B either K-major [N, K]
// (kBMn = false) or MN-major [K, N] (kBMn = true), both TMA-loaded.
template <bool kBMn, int kEpi>
__global__ void __launch_bounds__(kThreads, 1)
    bf16_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,  // A [M, K], box {64, 128}
                     const __grid_constant__ CUtensorMap tm_b,  // K-major: [N, K] box {64, 128}; MN-major: [K, N] box {64, 64}
                     const Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* as = smem;                               // kStages x 16 KiB
  uint8_t* bs = as + kStages * kABytes;             // kStages x 16 KiB
  Bars* bars = reinterpret_cast<Bars*>(bs + kStages * kBBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
  const int M = args.M, N = args.N, K = args.K;
  const int num_m = (M + 2 * kHalf - 1) / (2 * kHalf);
  const int num_n = (N + 2 * kHalf - 1) / (2 * kHalf);
  const int n_tiles = num_m * num_n;
  const int n_k = (K + kStageK - 1) / kStageK;
  volatile uint32_t* abort_word = &bars->abort_word;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->pfull[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->accum[b], 1);
      mbar_init(&bars->acc_empty[b], 2 * kEpiWarps);
    }
    bars->abort_word = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc2(&bars->tmem_base, kTmemCols);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      int g = 0;
      bool ok = true;
      for (int t = pair; t < n_tiles && ok; t += num_pairs) {
        const Tile tile = tile_at(t, num_m, num_n);
        const int mh = tile.m0 + static_cast<int>(crank) * kHalf;
        const int nh = tile.n0 + static_cast<int>(crank) * kHalf;
        for (int kt = 0; kt < n_k; ++kt, ++g) {
          const int s = g % kStages;
          if (g >= kStages &&
              !mbar_wait(&bars->empty[s], ((g / kStages) - 1) & 1, abort_word, args.status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bars->full[s], kABytes + kBBytes);
          tma_load_2d(as + s * kABytes, &tm_a, kt * kStageK, mh, &bars->full[s]);
          if constexpr (kBMn) {
            tma_load_2d(bs + s * kBBytes, &tm_b, nh, kt * kStageK, &bars->full[s]);
            tma_load_2d(bs + s * kBBytes + kBBytes / 2, &tm_b, nh + 64, kt * kStageK, &bars->full[s]);
          } else {
            tma_load_2d(bs + s * kBBytes, &tm_b, kt * kStageK, nh, &bars->full[s]);
          }
        }
      }
      for (int i = g > kStages ? g - kStages : 0; i < g; ++i) {
        uint32_t dummy = 0;
        mbar_wait(&bars->full[i % kStages], (i / kStages) & 1, &dummy, args.status, kStatusTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (crank == 0) {
      // ---------------------------------------------------- MMA issuer (leader)
      if (lane == 0) {
        const uint32_t idesc = kBMn ? idesc_bf16_f32_bmn(2 * kHalf, 2 * kHalf) : idesc_bf16_f32(2 * kHalf, 2 * kHalf);
        int g = 0, tl = 0;
        bool ok = true;
        for (int t = pair; t < n_tiles && ok; t += num_pairs, ++tl) {
          const int b = tl & 1;
          if (tl >= 2 && !mbar_wait_cluster(&bars->acc_empty[b], ((tl >> 1) - 1) & 1, abort_word, args.status,
                                            kStatusTimeoutAccum))
            break;
          tc_fence_after();
          const uint32_t acc = tmem_base + b * kAccCols;
          for (int kt = 0; kt < n_k; ++kt, ++g) {
            const int s = g % kStages;
            const uint32_t ph = (g / kStages) & 1;
            // Both CTAs' operand halves must have landed.
            if (!mbar_wait(&bars->full[s], ph, abort_word, args.status, kStatusTimeoutFull) ||
                !mbar_wait_cluster(&bars->pfull[s], ph, abort_word, args.status, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t adesc = sdesc_kmajor_sw128(smem_u32(as + s * kABytes));
            const uint64_t bdesc = kBMn ? sdesc_mnmajor_sw128(smem_u32(bs + s * kBBytes), kBBytes / 2, 1024)
                                        : sdesc_kmajor_sw128(smem_u32(bs + s * kBBytes));
            for (int kk = 0; kk < kStageK / 16; ++kk)
              mma_ss2(acc, adesc + 2 * kk, bdesc + (kBMn ? ((2 * 1024) >> 4) * kk : 2 * kk), idesc,
                      (kt | kk) != 0 ? 1u : 0u);
            tc_commit2_mc(&bars->empty[s], 0x3);
          }
          tc_commit2_mc(&bars->accum[b], 0x3);
        }
        if (tl > 0) {
          uint32_t dummy = 0;
          const int last = tl - 1;
          mbar_wait(&bars->accum[last & 1], (last >> 1) & 1, &dummy, args.status, kStatusTimeoutAccum);
        }
      }
    } else {
      // ------------------------------------------------- relay (peer CTA)
      // Tells the leader when this CTA's operand halves of each stage landed.
      if (lane == 0) {
        const uint32_t pfull_leader = mapa_shared(smem_u32(&bars->pfull[0]), 0);
        int g = 0;
        bool ok = true;
        for (int t = pair; t < n_tiles && ok; t += num_pairs)
          for (int kt = 0; kt < n_k; ++kt, ++g) {
            const int s = g % kStages;
            if (!mbar_wait(&bars->full[s], (g / kStages) & 1, abort_word, args.status, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            mbar_arrive_cluster(pfull_leader + s * 8);
          }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Lane quarter q (= warp & 3) holds this CTA's tokens mh + 32q + lane;
    // every thread walks the 256 columns of its row in 32-wide chunks.
    const int quarter = warp & 3;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(&bars->acc_empty[0]), 0);
    bool ok = true;
    int tl = 0;
    for (int t = pair; t < n_tiles; t += num_pairs, ++tl) {
      const Tile tile = tile_at(t, num_m, num_n);
      const int b = tl & 1;
      const int m = tile.m0 + static_cast<int>(crank) * kHalf + quarter * 32 + lane;
      float rmax = -INFINITY, rsum = 0.f;
      int tcol = -1;
      if constexpr (kEpi == kEpiCE) {
        if (m < M) {
          const int64_t tv = args.targets[m];
          if (tv != kIgnore && tv >= tile.n0 && tv < tile.n0 + 2 * kHalf) tcol = static_cast<int>(tv - tile.n0);
        }
      }
      if (ok && mbar_wait_warp(&bars->accum[b], (tl >> 1) & 1, abort_word, args.status, kStatusTimeoutAccum)) {
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < kAccCols; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem_base + b * kAccCols + lane_addr + c, v);
          tmem_wait_ld();
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) w[j] = pack_bf16x2(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
          const int n = tile.n0 + c;
          if (m < M && n < N) {
            __nv_bfloat16* dst = args.out + static_cast<size_t>(m) * args.ldo + n;
            if (n + 32 <= N) {
#pragma unroll
              for (int q = 0; q < 4; ++q)
                reinterpret_cast<uint4*>(dst)[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < N - n) reinterpret_cast<uint16_t*>(dst)[j] = static_cast<uint16_t>(w[j >> 1] >> (16 * (j & 1)));
            }
          }
          if constexpr (kEpi == kEpiCE) {
            // Online (max, sum exp) over the bf16-rounded logits of the chunk.
            const int live = min(32, N - n);
            float x[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) x[j] = __uint_as_float((w[j >> 1] >> (16 * (j & 1))) << 16);
            float cmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < live) cmax = fmaxf(cmax, x[j]);
            if (live > 0) {
              const float nmax = fmaxf(rmax, cmax);
              float s = rsum * __expf(rmax - nmax);
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < live) s += __expf(x[j] - nmax);
              rmax = nmax;
              rsum = s;
            }
            if (tcol >= c && tcol < c + 32 && m < M) {
              float tv = 0.f;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j == tcol - c) tv = x[j];
              args.tgt[m] = tv;
            }
          }
        }
        tc_fence_before();
        if constexpr (kEpi == kEpiCE) {
          if (m < M) args.part[static_cast<size_t>(m) * num_n + tile.n0 / (2 * kHalf)] = make_float2(rmax, rsum);
        }
      } else {
        ok = false;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader + b * 8);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc2(tmem_base, kTmemCols);
  }
}

// A target the loss reads: in [0, V).  kIgnore rows add nothing; any other
// value is invalid (F.cross_entropy raises for it): the row adds nothing, its
// dlogits are zero and kStatusBadInput is set.
__device__ __forceinline__ bool valid_target(int64_t t, int V) { return t >= 0 && t < V; }

// Row combine: lse[m] = max + log(sum s_i exp(max_i - max)); loss += lse - target
// logit for rows with a valid target.
__global__ void ce_rows_kernel(const float2* __restrict__ part, int n_tiles, const int64_t* __restrict__ targets,
                               const float* __restrict__ tgt, int M, int V, float* __restrict__ lse,
                               float* __restrict__ loss, uint32_t* __restrict__ status) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  const float2* p = part + static_cast<size_t>(warp) * n_tiles;
  float mx = -INFINITY;
  for (int i = lane; i < n_tiles; i += 32) mx = fmaxf(mx, p[i].x);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s = 0.f;
  for (int i = lane; i < n_tiles; i += 32) s += p[i].y * __expf(p[i].x - mx);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    const float l = mx + __logf(s);
    lse[warp] = l;
    const int64_t t = targets[warp];
    if (valid_target(t, V))
      atomicAdd(loss, l - tgt[warp]);
    else if (t != kIgnore)
      atomicOr(status, kStatusBadInput);
  }
}

// dlogits in place: (exp(x - lse) - [v == target]) * inv_norm, zero for
// ignored and invalid-target rows; rounded to bf16.
__global__ void dlogits_kernel(__nv_bfloat16* __restrict__ logits, int M, int V, const float* __restrict__ lse,
                               const int64_t* __restrict__ targets, float inv_norm) {
  const int64_t per_row = V / 8;  // 8 bf16 per vector (V % 8 == 0)
  const int64_t total = static_cast<int64_t>(M) * per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / per_row);
    const int v0 = static_cast<int>(i % per_row) * 8;
    const int64_t tv = targets[m];
    uint4* p = reinterpret_cast<uint4*>(logits + static_cast<size_t>(m) * V + v0);
    if (!valid_target(tv, V)) {
      *p = make_uint4(0, 0, 0, 0);
      continue;
    }
    const float l = lse[m];
    uint4 x = *p;
    uint32_t* w = reinterpret_cast<uint32_t*>(&x);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a = __uint_as_float(w[j] << 16), b = __uint_as_float(w[j] & 0xFFFF0000u);
      a = __expf(a - l) - (v0 + 2 * j == tv ? 1.f : 0.f);
      b = __expf(b - l) - (v0 + 2 * j + 1 == tv ? 1.f : 0.f);
      w[j] = pack_bf16x2(a * inv_norm, b * inv_norm);
    }
    *p = x;
  }
}

template <bool kBMn, int kEpi>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, cudaStream_t stream) {
  const int num_m = (a.M + 2 * kHalf - 1) / (2 * kHalf), num_n = (a.N + 2 * kHalf - 1) / (2 * kHalf);
  int pairs = 0;
  int rc = resident_pairs(reinterpret_cast<const void*>(&bf16_gemm_kernel<kBMn, kEpi>), kThreads, kSmemBytes, &pairs);
  if (rc) return rc;
  if (pairs > num_m * num_n) pairs = num_m * num_n;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
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
  cudaError_t le = cudaLaunchKernelEx(&cfg, bf16_gemm_kernel<kBMn, kEpi>, ta, tb, a);
  if (le != cudaSuccess) return set_error(FL_ERR_CUDA, "head gemm launch: %s", cudaGetErrorString(le));
  return FL_OK;
}

}  // namespace hd

// Workspace of one chunk: logits/dlogits bf16 [T, V], partials [T, ceil(V/256)]
// (max, sum), lse [T], target logits [T].
size_t ce_workspace_bytes(int64_t T, int64_t V) {
  const int64_t nt = (V + 255) / 256;
  auto a16 = [](size_t b) { return (b + 255) / 256 * 256; };
  return a16(static_cast<size_t>(T) * V * 2) + a16(static_cast<size_t>(T) * nt * 8) + 2 * a16(static_cast<size_t>(T) * 4);
}

int launch_ce_chunk(const void* h, int T, int H, const void* head, int V, const int64_t* targets, float inv_norm,
                    float* loss_sum, void* dh, void* ws, cudaStream_t stream) {
  using namespace hd;
  const int nt = (V + 255) / 256;
  auto a16 = [](size_t b) { return (b + 255) / 256 * 256; };
  uint8_t* w = static_cast<uint8_t*>(ws);
  auto* logits = reinterpret_cast<__nv_bfloat16*>(w);
  w += a16(static_cast<size_t>(T) * V * 2);
  auto* part = reinterpret_cast<float2*>(w);
  w += a16(static_cast<size_t>(T) * nt * 8);
  float* lse = reinterpret_cast<float*>(w);
  w += a16(static_cast<size_t>(T) * 4);
  float* tgt = reinterpret_cast<float*>(w);
  int dev = 0;
  cudaGetDevice(&dev);
  uint32_t* status = status_word(dev);
  if (!status) return set_error(FL_ERR_CUDA, "fl_ce_chunk: status word unavailable on device %d", dev);

  // 1. logits = h . head^T with the CE partials
  CUtensorMap ta, tb;
  int rc = make_tensor_map_2d(&ta, h, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, T, static_cast<uint64_t>(H) * 2, kStageK,
                              kHalf, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tensor_map_2d(&tb, head, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, V, static_cast<uint64_t>(H) * 2, kStageK,
                          kHalf, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  Args a{};
  a.out = logits;
  a.ldo = V;
  a.status = status;
  a.M = T;
  a.N = V;
  a.K = H;
  a.targets = targets;
  a.part = part;
  a.tgt = tgt;
  if ((rc = launch_gemm<false, kEpiCE>(ta, tb, a, stream))) return rc;
  // 2. rows
  ce_rows_kernel<<<(T * 32 + 255) / 256, 256, 0, stream>>>(part, nt, targets, tgt, T, V, lse, loss_sum, status);
  // 3. dlogits in place
  {
    const int64_t total = static_cast<int64_t>(T) * (V / 8);
    int64_t grid = (total + 255) / 256;
    if (grid > 148 * 16) grid = 148 * 16;
    dlogits_kernel<<<static_cast<int>(grid), 256, 0, stream>>>(logits, T, V, lse, targets, inv_norm);
  }
  // 4. dh = dlogits . head (head [V, H] is the MN-major B operand)
  rc = make_tensor_map_2d(&ta, logits, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, V, T, static_cast<uint64_t>(V) * 2, kStageK,
                          kHalf, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tensor_map_2d(&tb, head, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, H, V, static_cast<uint64_t>(H) * 2, 64, kStageK,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  Args d{};
  d.out = static_cast<__nv_bfloat16*>(dh);
  d.ldo = H;
  d.status = status;
  d.M = T;
  d.N = H;
  d.K = V;
  if ((rc = launch_gemm<true, kEpiStore>(ta, tb, d, stream))) return rc;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "ce chunk: %s", cudaGetErrorString(e));
  return FL_OK;
}

}  // namespace fl

using namespace fl;

extern "C" {

size_t fl_ce_workspace_bytes(int64_t T, int64_t V) {
  if (T <= 0 || V <= 0) return 0;
  return ce_workspace_bytes(T, V);
}

int fl_ce_chunk(const uint16_t* h, int64_t T, int64_t H, const uint16_t* head, int64_t V, const int64_t* targets,
                float inv_norm, float* loss_sum, uint16_t* dh, void* workspace, size_t workspace_bytes, void* stream) {
  if (T <= 0 || H <= 0 || V <= 0) return set_error(FL_ERR_ARG, "fl_ce_chunk: dims must be positive");
  if (T > (1 << 24) || H > (1 << 20) || V > (1 << 24)) return set_error(FL_ERR_ARG, "fl_ce_chunk: dims too large");
  if (H % 8 != 0 || V % 8 != 0)
    return set_error(FL_ERR_ARG, "fl_ce_chunk: hidden size and vocabulary must be multiples of 8");
  if (!h || !head || !targets || !loss_sum || !dh) return set_error(FL_ERR_ARG, "fl_ce_chunk: null pointer");
  if ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(head) | reinterpret_cast<uintptr_t>(dh)) & 15u)
    return set_error(FL_ERR_ARG, "fl_ce_chunk: h, head and dh must be 16-byte aligned");
  if (!(inv_norm > 0.0f) || inv_norm != inv_norm) return set_error(FL_ERR_ARG, "fl_ce_chunk: normalization must be > 0");
  if (!workspace || workspace_bytes < ce_workspace_bytes(T, V) || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return set_error(FL_ERR_ARG, "fl_ce_chunk: workspace missing, short or not 256-byte aligned");
  return launch_ce_chunk(h, (int)T, (int)H, head, (int)V, targets, inv_norm, loss_sum, dh, workspace,
                         static_cast<cudaStream_t>(stream));
}

}  // extern "C"
