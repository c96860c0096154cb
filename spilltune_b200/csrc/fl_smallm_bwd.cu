// Small-M backward of the frozen projection (M <= 16 tokens: decode-like steps):
//
//   dX[m, k] = sum_n dY[m, n] * W[n, k]  +  sum_j Us[m, j] * A[j, k],
//   W[n, k]  = bf16(lut[code[n, k]] * scale[n, k / 128]),   Us = bf16(s * dY . B)
//
// The tile GEMM's 256-token tiles leave most of the GPU idle here (one token
// tile: K/256 CTA pairs, each walking the whole reduction over n), so decode
// steps get their own kernel, the transpose of the small-M forward:
//   * The dX columns k are the MMA's M side: a CTA owns one 128-wide scale group
//     of columns (eight warps, 16 columns each) over a cluster slice of the
//     reduction over the weight rows n; the tokens are the 8-wide N dimension
//     of warp MMAs (mma.sync m16n8k16).
//   * Each 64-row chunk arrives in a ring slot by TMA: the codes of the CTA's
//     columns (64 B per row, 64-byte swizzle), dY for those rows (128-byte
//     swizzle, token rows past M zero-filled) and the rows' scales.  A producer
//     warp refills a slot once all consumer warps released it.
//   * Decode: the per-lane 256-entry byte table of the small-M forward gives the
//     bf16 pair of two adjacent columns of one row; movmatrix transposes each
//     8x8 block so a register holds two adjacent rows of one column — the MMA's
//     A fragment with the reduction over n.
//   * The scale varies along the reduction (one per row and group), so it goes
//     into the B operand: bf16(dY[m, n] * scale[n, group]) — one bf16 rounding
//     of dY * scale in place of the dequant's rounding of lut * scale.
// The CTAs of a cluster add their partial sums through distributed shared
// memory in rank order (deterministic); each finishes a slice of the columns:
// + Us . A in fp32, bf16 store.  The LoRA branch comes along in the epilogue:
// Us = bf16(s * dY . B) and Ts = bf16(s * X . A^T) are summed in a fixed order
// from the FP32 partials of the small-M low-rank kernels launched just before
// (the last of which lets this grid start early: programmatic dependent
// launch, so only the epilogue waits for them); each CTA then writes
// dA[:, its columns] = Us^T . X and dB for its share of the rows n = dY^T . Ts
// (every element by one thread, so no atomics).
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {

int make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);

namespace smb {

constexpr int kCols = 128;                        // dX columns (W columns) per CTA: one scale group
constexpr int kChunkN = 64;                       // reduction rows (W rows) per ring slot
constexpr int kWarps = 8;                         // consumer warps, 16 columns each
constexpr int kThreads = 32 * (kWarps + 1);       // + one TMA producer warp
constexpr int kTableBytes = 256 * 256;           // [byte][256-byte row: lane] bf16 pairs
constexpr int kCodeBytes = kChunkN * kCols / 2;   // 64 rows x 64 B
constexpr int kScaleBytes = kChunkN * 16;         // 64 rows x 4 groups (fp32)
constexpr int kRedBytes = kCols * 16 * 4;         // fp32 partial dX [column][16 tokens]
constexpr int kMaxSplit = 8;
constexpr int kUsStride = 65;                     // fp32 Us rows, padded against bank conflicts
__host__ __device__ constexpr int dy_bytes(int nt) { return 8 * nt * 128; }  // [8 NT tokens][64 n] bf16
__host__ __device__ constexpr int slot_bytes(int nt) { return kCodeBytes + dy_bytes(nt) + kScaleBytes; }
__host__ __device__ constexpr int slot_stride(int nt) { return (slot_bytes(nt) + 1023) / 1024 * 1024; }
// Ring depth: the most slots that keep two CTAs per SM next to the 64 KiB table.
__host__ __device__ constexpr int slots_of(int nt) { return nt == 2 ? 5 : 6; }
// Dynamic shared memory: table (at offset 0: a constant address) | ring | partial dX |
// full and empty mbarriers + abort word.
__host__ __device__ constexpr int smem_bytes(int nt) {
  return kTableBytes + 1024 + slots_of(nt) * slot_stride(nt) + kRedBytes + 2 * slots_of(nt) * 8 + 16;
}
static_assert(2 * (smem_bytes(1) + 1024) <= 233472 && 2 * (smem_bytes(2) + 1024) <= 233472, "two CTAs per SM");
// After the main loop the table's space holds A columns [rank][128] and the
// ring's space Us, Ts [16][kUsStride] and X columns [16][128] (fp32).
static_assert(64 * kCols * 4 <= kTableBytes, "A staging");
static_assert((2 * 16 * kUsStride + 16 * kCols) * 4 <= slots_of(2) * kCodeBytes, "Us, Ts, X staging");

struct Args {
  const __nv_bfloat16* dY;  // [M, N]
  const __nv_bfloat16* X;   // [M, K] (rank > 0)
  const float* uparts;      // [M][64][n_uparts] partials of dY . B (rank > 0)
  const float* tparts;      // [M][64][n_tparts] partials of X . A^T (rank > 0)
  int n_uparts, n_tparts;
  float s;                  // LoRA scale
  const float* lut;         // [16]
  const float* alora;       // [rank, K]
  __nv_bfloat16* dX;        // [M, K]
  float* dA;                // [rank, K]
  float* dB;                // [N, rank]
  int accumulate;           // dA, dB += (else =)
  uint32_t* status;
  int M, N, K, rank;
  int split;                // CTAs of a cluster along the reduction
};

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bf16x2 {lo, hi} -> bf16x2 {bf16(lo * s0), bf16(hi * s1)}
__device__ __forceinline__ uint32_t scale_pair(uint32_t v, float s0, float s1) {
  return pack_bf16x2(__uint_as_float(v << 16) * s0, __uint_as_float(v & 0xFFFF0000u) * s1);
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 2)
    smallm_bwd_kernel(const __grid_constant__ CUtensorMap tm_codes,   // [N, K/2] u8, box {64, 64}, 64-byte swizzle
                      const __grid_constant__ CUtensorMap tm_dy,      // [M, N] bf16, box {64, 8 NT}, 128-byte swizzle
                      const __grid_constant__ CUtensorMap tm_scales,  // [N, K/128] fp32, box {4, 64}
                      const Args args) {
  extern __shared__ uint8_t smem_raw[];
  constexpr int kSlots = slots_of(NT);
  constexpr int sbytes = slot_stride(NT);
  constexpr int kDyOff = kCodeBytes;
  constexpr int kSOff = kCodeBytes + dy_bytes(NT);
  uint8_t* table = smem_raw;
  uint8_t* ring = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + kTableBytes + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(ring + kSlots * sbytes);                // [column][16]
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + kRedBytes);
  uint64_t* empty = full + kSlots;
  volatile uint32_t* abort_word = reinterpret_cast<volatile uint32_t*>(empty + kSlots);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c4 = lane & 3;
  const int split = args.split;
  const int kslice = split > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int cb = blockIdx.x / split;  // column block = scale group
  const int k0 = cb * kCols;
  const int chunks = args.N / kChunkN;
  const int c_begin = kslice * chunks / split;
  const int n_ch = (kslice + 1) * chunks / split - c_begin;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tm_codes);
    tma_prefetch_desc(&tm_dy);
    tma_prefetch_desc(&tm_scales);
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWarps);
    }
    *abort_word = 0;
    fence_barrier_init();
  }
  auto issue = [&](int k) {  // chunk c_begin + k into slot k % kSlots (one thread)
    const int sl = k % kSlots;
    uint8_t* dst = ring + sl * sbytes;
    const int n0 = (c_begin + k) * kChunkN;
    mbar_arrive_expect_tx(&full[sl], slot_bytes(NT));
    tma_load_2d(dst, &tm_codes, k0 / 2, n0, &full[sl]);
    tma_load_2d(dst + kDyOff, &tm_dy, n0, 0, &full[sl]);
    tma_load_2d(dst + kSOff, &tm_scales, (cb / 4) * 4, n0, &full[sl]);
  };
  __syncthreads();  // barriers initialised
  if (threadIdx.x == 0)
    for (int i = 0; i < kSlots && i < n_ch; ++i) issue(i);
  // Per-lane byte table: entry e of lane l at table + 256 e + 4 l holds the
  // bf16 pair {lut[e & 15], lut[e >> 4]} (the upper half of each 256-byte
  // row stays unused: one byte permute then forms a lookup's whole address).
  if (warp < kWarps) {
    const float mine = __ldg(args.lut + (lane & 15));
    const int e = 32 * warp + lane;
    const uint32_t packed =
        pack_bf16x2(__shfl_sync(0xffffffffu, mine, e & 15), __shfl_sync(0xffffffffu, mine, e >> 4));
    uint32_t* tw = reinterpret_cast<uint32_t*>(table) + 32 * warp * 64 + lane;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) tw[j * 64] = __shfl_sync(0xffffffffu, packed, j);
  }
  __syncthreads();

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
  bool ok = true;
  if (warp == kWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int k = kSlots;
      for (; k < n_ch; ++k) {
        const int sl = k % kSlots;
        if (!mbar_wait(&empty[sl], ((k / kSlots) - 1) & 1, abort_word, args.status, kStatusTimeoutEmpty)) break;
        fence_proxy_async_smem();  // the consumers' generic reads before the async-proxy refill
        issue(k);
      }
      // Never leave the CTA with bulk copies still landing in its shared memory.
      const int issued = k < n_ch ? k : n_ch;
      for (int i = issued > kSlots ? issued - kSlots : 0; i < issued; ++i) {
        uint32_t dummy = 0;
        mbar_wait(&full[i % kSlots], (i / kSlots) & 1, &dummy, args.status, kStatusTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const uint32_t tab0 = smem_u32(table);
    const uint32_t lane4 = static_cast<uint32_t>(lane) * 4;
    // prmt selector giving {lane4 byte 0, byte c4 of the word, 0, 0}: the
    // lookup's offset (byte << 8) | 4 lane in one instruction.
    const uint32_t sel = 0x5504u | (static_cast<uint32_t>(c4) << 4);
    auto lookup = [&](uint32_t w) { return lds_u32(tab0 + prmt(w, lane4, sel)); };
    const int gcol = cb & 3;  // this CTA's group within the 4-group scale box
    for (int k = 0; k < n_ch && ok; ++k) {
      const int sl = k % kSlots;
      if (!mbar_wait_warp(&full[sl], (k / kSlots) & 1, abort_word, args.status, kStatusTimeoutFull)) {
        ok = false;
        break;
      }
      const uint8_t* slot = ring + sl * sbytes;
      const float* scl = reinterpret_cast<const float*>(slot + kSOff);
#pragma unroll
      for (int ns = 0; ns < kChunkN / 16; ++ns) {
        // This warp's 8 code bytes (columns 16 warp .. +15) of rows 16 ns + g and +8:
        // 16-byte chunk warp / 2 of the 64-byte row, moved by the 64-byte swizzle.
        const int r0 = 16 * ns + g, r1 = r0 + 8;
        const uint2 q0 = *reinterpret_cast<const uint2*>(slot + r0 * 64 + (((warp >> 1) ^ ((r0 >> 1) & 3)) << 4) +
                                                         ((warp & 1) << 3));
        const uint2 q1 = *reinterpret_cast<const uint2*>(slot + r1 * 64 + (((warp >> 1) ^ ((r1 >> 1) & 3)) << 4) +
                                                         ((warp & 1) << 3));
        // 8x8 blocks [row n][column k] -> transposed A fragments [column][row].
        const uint32_t a0 = movmatrix_trans(lookup(q0.x));  // columns 0-7,  rows 0-7
        const uint32_t a1 = movmatrix_trans(lookup(q0.y));  // columns 8-15, rows 0-7
        const uint32_t a2 = movmatrix_trans(lookup(q1.x));  // columns 0-7,  rows 8-15
        const uint32_t a3 = movmatrix_trans(lookup(q1.y));  // columns 8-15, rows 8-15
        // B: dY * scale for rows 16 ns + 2 c4 + {0, 1} (b0) and + 8 (b1).
        const int rn = 16 * ns + 2 * c4;
        const float s0 = scl[rn * 4 + gcol], s1 = scl[(rn + 1) * 4 + gcol];
        const float s2 = scl[(rn + 8) * 4 + gcol], s3 = scl[(rn + 9) * 4 + gcol];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          // dY row 8 nt + g: 16-byte chunks 2 ns and 2 ns + 1 of its 128-byte row (swizzled by g).
          const uint8_t* dyr = slot + kDyOff + (8 * nt + g) * 128 + 4 * c4;
          const uint32_t d0 = *reinterpret_cast<const uint32_t*>(dyr + (((2 * ns) ^ g) << 4));
          const uint32_t d1 = *reinterpret_cast<const uint32_t*>(dyr + (((2 * ns + 1) ^ g) << 4));
          mma16816(acc[nt], a0, a1, a2, a3, scale_pair(d0, s0, s1), scale_pair(d1, s2, s3));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[sl]);
    }
    // Partial dX: accumulator element i: column 16 warp + g + 8 (i >> 1), token 8 nt + 2 c4 + (i & 1).
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[(16 * warp + g + 8 * (i >> 1)) * 16 + 8 * nt + 2 * c4 + (i & 1)] = acc[nt][i];
  }
  __syncthreads();
  if (split > 1) cluster_sync();

  // Columns [kc0, kc0 + cols) of the block: the cluster's partials in rank order
  // + Us . A, bf16 store.
  const int cols = kCols / split;
  const int kc0 = kslice * cols;
  float* al = reinterpret_cast<float*>(table);  // A [j][column of the block]
  float* us = reinterpret_cast<float*>(ring);   // Us [token][kUsStride]
  float* ts = us + 16 * kUsStride;              // Ts [token][kUsStride]
  float* xs = ts + 16 * kUsStride;              // X [token][column of the block]
  if (args.rank > 0) {
    // Inputs that do not depend on the low-rank kernels first.
    for (int idx = threadIdx.x; idx < args.rank * cols; idx += kThreads) {
      const int j = idx / cols, c = kc0 + idx % cols;
      al[j * kCols + c] = __ldg(args.alora + static_cast<size_t>(j) * args.K + k0 + c);
    }
    for (int idx = threadIdx.x; idx < args.M * cols; idx += kThreads) {
      const int m = idx / cols, c = kc0 + idx % cols;
      xs[m * kCols + c] = __bfloat162float(args.X[static_cast<size_t>(m) * args.K + k0 + c]);
    }
    griddep_wait();
    // Us and Ts: bf16(s * the partials summed in order).
    for (int idx = threadIdx.x; idx < 2 * args.M * args.rank; idx += kThreads) {
      const bool is_t = idx >= args.M * args.rank;
      const int o = is_t ? idx - args.M * args.rank : idx;
      const int m = o / args.rank, j = o % args.rank;
      const int np = is_t ? args.n_tparts : args.n_uparts;
      const float* src = (is_t ? args.tparts : args.uparts) + (static_cast<size_t>(m) * 64 + j) * np;
      float v = 0.f;
#pragma unroll 4
      for (int c = 0; c < np; ++c) v += __ldg(src + c);
      (is_t ? ts : us)[m * kUsStride + j] = __bfloat162float(__float2bfloat16_rn(args.s * v));
    }
    __syncthreads();
  }
  const uint32_t red_local = smem_u32(red);
  for (int idx = threadIdx.x; idx < cols * args.M; idx += kThreads) {
    const int tok = idx / cols, c = kc0 + idx % cols;
    const int off = c * 16 + tok;
    float v = 0.f;
#pragma unroll
    for (int p = 0; p < kMaxSplit; ++p)
      if (p < split)
        v += p == kslice ? red[off]
                         : __uint_as_float(ld_shared_cluster_u32(mapa_shared(red_local, static_cast<uint32_t>(p)) +
                                                                 static_cast<uint32_t>(off) * 4));
    if (args.rank > 0) {
      const float* ur = us + tok * kUsStride;
      for (int j = 0; j < args.rank; ++j) v = fmaf(ur[j], al[j * kCols + c], v);
    }
    args.dX[static_cast<size_t>(tok) * args.K + k0 + c] = __float2bfloat16_rn(v);
  }
  if (args.rank > 0) {
    // dA[j, k] = sum_m Us[m, j] X[m, k] for this CTA's columns.
    for (int idx = threadIdx.x; idx < args.rank * cols; idx += kThreads) {
      const int j = idx / cols, c = kc0 + idx % cols;
      float v = 0.f;
      for (int m = 0; m < args.M; ++m) v = fmaf(us[m * kUsStride + j], xs[m * kCols + c], v);
      float* dst = args.dA + static_cast<size_t>(j) * args.K + k0 + c;
      *dst = args.accumulate ? *dst + v : v;
    }
    // dB[n, j] = sum_m dY[m, n] Ts[m, j] for rows n of this CTA's reduction
    // slice with (n - first row) % (column blocks) == column block.
    const int blocks = args.K / kCols;
    const int n_begin = c_begin * kChunkN, n_rows = n_ch * kChunkN;
    const int mine = (n_rows - cb + blocks - 1) / blocks;
    for (int i = threadIdx.x; i < mine; i += kThreads) {
      const int n = n_begin + cb + i * blocks;
      float dy[16];  // column n of dY, read once for every rank
#pragma unroll
      for (int m = 0; m < 16; ++m)
        dy[m] = m < args.M ? __bfloat162float(args.dY[static_cast<size_t>(m) * args.N + n]) : 0.f;
      float* dst = args.dB + static_cast<size_t>(n) * args.rank;
      for (int j = 0; j < args.rank; ++j) {
        float v = 0.f;
#pragma unroll
        for (int m = 0; m < 16; ++m)
          if (m < args.M) v = fmaf(dy[m], ts[m * kUsStride + j], v);  // rows past M of Ts are not staged
        dst[j] = args.accumulate ? dst[j] + v : v;
      }
    }
  }
  if (split > 1) cluster_sync();  // peers' partials stay valid until every CTA has read them
}

template <int NT>
static int launch_nt(const CUtensorMap& tc, const CUtensorMap& td, const CUtensorMap& ts, const Args& a, int blocks,
                     bool pdl, cudaStream_t stream) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&smallm_bwd_kernel<NT>),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(NT));
    if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "small-M backward attr: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks * a.split);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes(NT);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  cudaError_t le = cudaLaunchKernelEx(&cfg, smallm_bwd_kernel<NT>, tc, td, ts, a);
  if (le != cudaSuccess) return set_error(FL_ERR_CUDA, "small-M backward launch: %s", cudaGetErrorString(le));
  return FL_OK;
}

}  // namespace smb

int launch_smallm_bwd(const void* dY, const void* X, const float* uparts, const float* tparts, float s,
                      const uint8_t* codes, const float* scales, const float* lut, const float* alora, int rank,
                      void* dX, float* dA, float* dB, int accumulate, int M, int N, int K, cudaStream_t stream) {
  using namespace smb;
  if (M < 1 || M > 16 || K % 512 != 0 || N % kChunkN != 0)
    return set_error(FL_ERR_ARG, "small-M backward needs 1 <= M <= 16, K %% 512 == 0, N %% 64 == 0");
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    sms = 148;
  // One wave at two CTAs per SM: split the reduction over a cluster while the grid fits.
  const int blocks = K / kCols;
  const int chunks = N / kChunkN;
  int split = 1;
  while (split < kMaxSplit && blocks * split * 2 <= 2 * sms && chunks >= 2 * split) split *= 2;
  Args a;
  a.dY = static_cast<const __nv_bfloat16*>(dY);
  a.X = static_cast<const __nv_bfloat16*>(X);
  a.uparts = uparts;
  a.tparts = tparts;
  const int csize = lora_parts_per_cluster(K, N);  // the one launch_lora_parts2 made both with
  a.n_uparts = N / (128 * csize);
  a.n_tparts = K / (128 * csize);
  a.s = s;
  a.dA = dA;
  a.dB = dB;
  a.accumulate = accumulate;
  a.lut = lut;
  a.alora = alora;
  a.dX = static_cast<__nv_bfloat16*>(dX);
  a.status = status_word(dev);
  a.M = M;
  a.N = N;
  a.K = K;
  a.rank = rank;
  a.split = split;
  const int nt = M <= 8 ? 1 : 2;
  CUtensorMap tc, td, ts;
  int rc = make_tensor_map_2d(&tc, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, N, K / 2, kCols / 2, kChunkN,
                              CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  rc = make_tensor_map_2d(&td, dY, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, N, M, static_cast<uint64_t>(N) * 2, 64, 8 * nt,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tensor_map_2d(&ts, scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, K / 128, N, static_cast<uint64_t>(K / 128) * 4,
                          4, kChunkN, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  // With a LoRA branch the preceding launch wrote the last partials: start while it runs.
  const bool pdl = rank > 0;
  if (nt == 1) return launch_nt<1>(tc, td, ts, a, blocks, pdl, stream);
  return launch_nt<2>(tc, td, ts, a, blocks, pdl, stream);
}

}  // namespace fl
