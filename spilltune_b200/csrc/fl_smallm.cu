// Small-M frozen projection (M <= 16 tokens: decode-like steps):
//
//   Y[m, n] = sum_g scale[n, g] * sum_{k in g} X[m, k] * L[code[n, k]]  +  sum_j Ts[m, j] * Blora[n, j]
//
// the same product as fl_fwd with each 128-wide scale group factored out of
// its dot product, so the tensor-core operand is L = bf16(lut) — exactly the
// stored code for int4-sym (c - 8), the bf16-rounded codebook for NF4 — and the
// scale multiplies the fp32 partial sum of its group.
//
// At M <= 16 every weight byte is used once and a whole projection is only a
// few MB, so the kernel is bound by how fast the packed weights can be put in
// flight: each CTA owns 16*tpc weight rows over the whole reduction (or one
// cluster slice of it) and, before anything else, queues TMA loads of its
// first `slots` 512-column chunks (codes with the 128-byte swizzle, plus the
// chunk's scales) into a ring of shared-memory slots; the grid is one wave of
// several small CTAs per SM, so decode latency is hidden by other warps.
// Decode: the 16 operand values bf16(lut[c]) sit in registers as a low-byte
// and a high-byte plane (the product table of fl_codebook.cuh with scale 1),
// and prmt looks up eight codes of a payload word at a time — no table to
// build in shared memory, no shared-memory lookups.  Four
// warps each take one 128-wide scale group of every chunk; the MMAs are
// warp-level (mma.sync m16n8k16) with 16 weight rows as A and the tokens as
// the 8-wide N dimension, X fragments read from global (L2) one chunk ahead.
// The reduction-split CTAs of a cluster add their partial sums through
// distributed shared memory; rank 0 adds the LoRA term and writes Y.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_codebook.cuh"
#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {

int make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);

namespace sm {

constexpr int kWarps = 4;                        // one per 128-wide group of a chunk
constexpr int kThreads = 32 * kWarps;
constexpr int kChunkK = 512;                     // reduction columns per ring slot
constexpr int kMaxTpc = 8;                       // 16-row tiles per CTA
constexpr int kCtasPerSm = 3;                    // grid = one wave at this many CTAs per SM (registers allow 3)
constexpr int kSlotBudget = 40 * 1024;           // ring bytes per CTA

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t word4(const uint4& q, int w) {
  return w == 0 ? q.x : w == 1 ? q.y : w == 2 ? q.z : q.w;
}

struct Args {
  const __nv_bfloat16* X;   // [M, K]
  const __nv_bfloat16* Ts;  // [M, 64] scaled low-rank activations (rank > 0)
  const float* lut;         // [16]
  const float* blora;       // [N, rank]
  __nv_bfloat16* Y;         // [M, N]
  uint32_t* status;
  int M, N, K, rank;
  int tpc;                  // 16-row tiles per CTA
  int split;                // CTAs of a cluster along the reduction
  int slots;                // ring depth
};

// Slot layout: codes box 0 (columns 0..255 of the chunk) [rows][128 B],
// codes box 1 (256..511), scales [rows][4 fp32].
__host__ __device__ constexpr int slot_bytes(int rows) { return rows * 128 * 2 + rows * 16; }

// NT: 8-token tiles, 1 (M <= 8) or 2 (M <= 16).  TPC: 16-row tiles per CTA,
// unrolled so the MMA chains of different tiles interleave; with few tiles
// the k-steps alternate between two partial sums (PS = 2) for the same reason.
template <int NT, int TPC>
__global__ void __launch_bounds__(kThreads)
    smallm_kernel(const __grid_constant__ CUtensorMap tm_codes,   // [N, K/2] u8, box {128, rows}, 128B swizzle
                  const __grid_constant__ CUtensorMap tm_scales,  // [N, K/128] fp32, box {4, rows}
                  const Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int PS = TPC * NT <= 2 ? 2 : 1;
  const int rows = 16 * TPC;
  const int sbytes = (slot_bytes(rows) + 1023) / 1024 * 1024;
  uint8_t* ring = smem;                                                // slots x sbytes
  float* red = reinterpret_cast<float*>(smem + args.slots * sbytes);   // [kWarps][rows][16]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + kWarps * rows * 16);         // [slots], then the abort word
  volatile uint32_t* abort_word = reinterpret_cast<volatile uint32_t*>(full + args.slots);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c4 = lane & 3;
  const int split = args.split;
  const int kslice = split > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int n0 = (blockIdx.x / split) * rows;
  const int chunks = args.K / kChunkK;
  const int c_begin = kslice * chunks / split;
  const int c_end = (kslice + 1) * chunks / split;
  const int n_ch = c_end - c_begin;
  // Every CTA reads the same X: start each at a different chunk so the CTAs
  // spread over X instead of all asking the same L2 lines at once.
  const int rot = n_ch > 0 ? static_cast<int>((blockIdx.x / split) % n_ch) : 0;
  auto chunk_of = [&](int k) { return c_begin + (k + rot) % n_ch; };

  // Queue the first loads before any other work.
  if (threadIdx.x == 0) {
    for (int i = 0; i < args.slots; ++i) mbar_init(&full[i], 1);
    *abort_word = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_codes);
    tma_prefetch_desc(&tm_scales);
  }
  auto issue = [&](int k) {  // chunk c_begin + k into slot k % slots (thread 0)
    const int sl = k % args.slots;
    uint8_t* dst = ring + sl * sbytes;
    const int c = chunk_of(k);
    mbar_arrive_expect_tx(&full[sl], slot_bytes(rows));
    tma_load_2d(dst, &tm_codes, c * (kChunkK / 2), n0, &full[sl]);
    tma_load_2d(dst + rows * 128, &tm_codes, c * (kChunkK / 2) + 128, n0, &full[sl]);
    tma_load_2d(dst + rows * 256, &tm_scales, c * 4, n0, &full[sl]);
  };
  int issued = 0;  // meaningful in thread 0 only
  if (threadIdx.x == 0)
    for (; issued < args.slots && issued < n_ch; ++issued) issue(issued);
  // Operand table bf16(lut[c]) in registers.
  const ProductTable table = make_table(args.lut, 1.0f);
  __syncthreads();

  float acc[TPC][NT][4];
#pragma unroll
  for (int t = 0; t < TPC; ++t)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[t][nt][0] = acc[t][nt][1] = acc[t][nt][2] = acc[t][nt][3] = 0.f;

  // X fragments of chunk c for this warp's group: tokens g (+8), columns
  // 512c + 128*warp + 32*c4 + [0, 32) — 64 contiguous bytes per token.
  auto load_x = [&](int c, uint4 (&xv)[NT][4]) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int tok = 8 * nt + g;
      const uint4* src = reinterpret_cast<const uint4*>(args.X + static_cast<size_t>(tok < args.M ? tok : 0) * args.K +
                                                        c * kChunkK + 128 * warp + 32 * c4);
#pragma unroll
      for (int i = 0; i < 4; ++i) xv[nt][i] = tok < args.M ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
    }
  };

  // One chunk: wait for its slot, decode + MMA this warp's group for every
  // tile, then (all warps past the slot) refill it.  Every warp passes the
  // same __syncthreads whether or not a wait gave up.
  bool ok = true;
  auto chunk = [&](int k, const uint4 (&xv)[NT][4]) {
    const int sl = k % args.slots;
    if (ok && !mbar_wait_short_warp(&full[sl], (k / args.slots) & 1, abort_word, args.status, kStatusTimeoutFull))
      ok = false;
    if (ok) {
      const uint8_t* slot = ring + sl * sbytes;
      const uint8_t* cbox = slot + (warp >> 1) * rows * 128;  // this warp's group sits in box warp/2
      const int j = (warp & 1) * 4 + c4;                       // 16-byte chunk of the row in that box
      const float* scl = reinterpret_cast<const float*>(slot + rows * 256);
      uint4 q[TPC][2];
#pragma unroll
      for (int t = 0; t < TPC; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = 16 * t + g + 8 * h;
          q[t][h] = *reinterpret_cast<const uint4*>(cbox + r * 128 + ((j ^ (r & 7)) << 4));
        }
      float part[PS][TPC][NT][4];
#pragma unroll
      for (int p = 0; p < PS; ++p)
#pragma unroll
        for (int t = 0; t < TPC; ++t)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) part[p][t][nt][0] = part[p][t][nt][1] = part[p][t][nt][2] = part[p][t][nt][3] = 0.f;
      // Payload word w of the thread's 16 bytes holds columns 32c4 + 8w + [0, 8);
      // MMA k-step kk = 2w + s uses its pairs 2s (columns +4s+{0,1}) and 2s+1 (+{2,3}).
#pragma unroll
      for (int w = 0; w < 4; ++w) {
#pragma unroll
        for (int t = 0; t < TPC; ++t) {
          uint32_t e0[4], e1[4];  // rows g and g + 8
          lookup8(table, word4(q[t][0], w), e0);
          lookup8(table, word4(q[t][1], w), e1);
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            const int kk = 2 * w + sub;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint4& xq = xv[nt][w];
              const uint32_t b0 = sub ? xq.z : xq.x, b1 = sub ? xq.w : xq.y;
              mma16816(part[kk % PS][t][nt], e0[2 * sub], e1[2 * sub], e0[2 * sub + 1], e1[2 * sub + 1], b0, b1);
            }
          }
        }
      }
#pragma unroll
      for (int t = 0; t < TPC; ++t) {
        const int r0 = 16 * t + g, r1 = r0 + 8;
        const float s0 = scl[r0 * 4 + warp], s1 = scl[r1 * 4 + warp];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float v[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i] = PS == 2 ? part[0][t][nt][i] + part[PS - 1][t][nt][i] : part[0][t][nt][i];
          acc[t][nt][0] = fmaf(s0, v[0], acc[t][nt][0]);
          acc[t][nt][1] = fmaf(s0, v[1], acc[t][nt][1]);
          acc[t][nt][2] = fmaf(s1, v[2], acc[t][nt][2]);
          acc[t][nt][3] = fmaf(s1, v[3], acc[t][nt][3]);
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && issued < n_ch && !*abort_word) {
      fence_proxy_async_smem();  // the slot's generic reads before the async-proxy refill
      issue(issued);
      ++issued;
    }
  };
  uint4 xa[NT][4], xb[NT][4];
  if (n_ch > 0) load_x(chunk_of(0), xa);
  for (int k = 0; k < n_ch; k += 2) {
    if (k + 1 < n_ch) load_x(chunk_of(k + 1), xb);
    chunk(k, xa);
    if (k + 1 < n_ch) {
      if (k + 2 < n_ch) load_x(chunk_of(k + 2), xa);
      chunk(k + 1, xb);
    }
  }
  // After an abort, loads already queued may still land: wait for them
  // (bounded) before the shared memory is released.
  if (threadIdx.x == 0 && *abort_word) {
    for (int k = issued > args.slots ? issued - args.slots : 0; k < issued; ++k) {
      uint32_t dummy = 0;
      mbar_wait_short(&full[k % args.slots], (k / args.slots) & 1, &dummy, args.status, kStatusTimeoutDrain);
    }
  }

  // ------------------------------------------------------------ reductions
  // Warp partials -> red[warp][row][token]; accumulator element i of tile t:
  // row 16t + g + 8*(i >> 1), token 8*nt + 2*c4 + (i & 1).
#pragma unroll
  for (int t = 0; t < TPC; ++t) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        red[(warp * rows + 16 * t + g + 8 * (i >> 1)) * 16 + 8 * nt + 2 * c4 + (i & 1)] = acc[t][nt][i];
  }
  __syncthreads();
  // Sum the four group warps into red[0] (tokens past 8*NT stay unused).
  for (int idx = threadIdx.x; idx < rows * 16; idx += kThreads)
    red[idx] = red[idx] + red[rows * 16 + idx] + red[2 * rows * 16 + idx] + red[3 * rows * 16 + idx];
  if (split > 1) {
    cluster_sync();
  } else {
    __syncthreads();
  }
  if (kslice == 0) {
    const uint32_t red_local = smem_u32(red);
    for (int idx = threadIdx.x; idx < rows * 16; idx += kThreads) {
      const int lr = idx >> 4, tok = idx & 15;
      const int n = n0 + lr;
      if (n < args.N && tok < args.M) {
        float v = red[idx];
        for (int p = 1; p < split; ++p)
          v += __uint_as_float(ld_shared_cluster_u32(mapa_shared(red_local, static_cast<uint32_t>(p)) + idx * 4));
        if (args.rank > 0) {
          const __nv_bfloat16* tr = args.Ts + static_cast<size_t>(tok) * 64;
          const float* br = args.blora + static_cast<size_t>(n) * args.rank;
          for (int jj = 0; jj < args.rank; ++jj) v = fmaf(__bfloat162float(tr[jj]), __ldg(br + jj), v);
        }
        args.Y[static_cast<size_t>(tok) * args.N + n] = __float2bfloat16_rn(v);
      }
    }
  }
  if (split > 1) cluster_sync();  // peers' partials stay valid until rank 0 has read them
}

template <int NT, int TPC>
static int launch_nt(const Args& a, const CUtensorMap& tc, const CUtensorMap& ts, int blocks, int smem,
                     cudaStream_t stream) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&smallm_kernel<NT, TPC>),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "small-M attr: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks * a.split);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t le = cudaLaunchKernelEx(&cfg, smallm_kernel<NT, TPC>, tc, ts, a);
  if (le != cudaSuccess) return set_error(FL_ERR_CUDA, "small-M launch: %s", cudaGetErrorString(le));
  return FL_OK;
}

}  // namespace sm

int launch_smallm_fwd(const void* X, const void* Ts, const uint8_t* codes, const float* scales, const float* lut,
                      const float* lora, int rank, void* Y, int M, int N, int K, cudaStream_t stream) {
  using namespace sm;
  if (M < 1 || M > 16) return set_error(FL_ERR_ARG, "small-M path needs 1 <= M <= 16");
  if (K % kChunkK != 0) return set_error(FL_ERR_ARG, "small-M path needs K %% 512 == 0");
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    sms = 148;
  // One wave at kCtasPerSm CTAs per SM: the fewest 16-row tiles per CTA that
  // fit (1, 2, 4 or 8).
  const int tiles = (N + 15) / 16;
  const int want = (tiles + kCtasPerSm * sms - 1) / (kCtasPerSm * sms);
  int tpc = 1;
  const int max_tpc = M <= 8 ? kMaxTpc : kMaxTpc / 2;  // 16 tokens x 8 tiles would spill registers
  while (tpc < want && tpc < max_tpc) tpc *= 2;
  const int rows = 16 * tpc;
  const int blocks = (N + rows - 1) / rows;
  // Too few row blocks: split the reduction across a cluster.
  const int chunks = K / kChunkK;
  int split = 1;
  while (split < 8 && blocks * split * 2 <= kCtasPerSm * sms && chunks >= 2 * split) split *= 2;
  const int sbytes = (slot_bytes(rows) + 1023) / 1024 * 1024;
  int slots = kSlotBudget / sbytes;
  if (slots > 8) slots = 8;
  if (slots < 2) slots = 2;
  const int smem = 1024 + slots * sbytes + kWarps * rows * 16 * 4 + slots * 8 + 16;
  Args a;
  a.X = static_cast<const __nv_bfloat16*>(X);
  a.Ts = static_cast<const __nv_bfloat16*>(Ts);
  a.lut = lut;
  a.blora = lora;
  a.Y = static_cast<__nv_bfloat16*>(Y);
  a.status = status_word(dev);
  a.M = M;
  a.N = N;
  a.K = K;
  a.rank = rank;
  a.tpc = tpc;
  a.split = split;
  a.slots = slots;
  CUtensorMap tc, ts;
  int rc = make_tensor_map_2d(&tc, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, N, K / 2, 128, rows,
                              CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tensor_map_2d(&ts, scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, K / 128, N, static_cast<uint64_t>(K / 128) * 4,
                          4, rows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (M <= 8) {
    if (tpc == 1) return launch_nt<1, 1>(a, tc, ts, blocks, smem, stream);
    if (tpc == 2) return launch_nt<1, 2>(a, tc, ts, blocks, smem, stream);
    if (tpc == 4) return launch_nt<1, 4>(a, tc, ts, blocks, smem, stream);
    return launch_nt<1, 8>(a, tc, ts, blocks, smem, stream);
  }
  if (tpc == 1) return launch_nt<2, 1>(a, tc, ts, blocks, smem, stream);
  if (tpc == 2) return launch_nt<2, 2>(a, tc, ts, blocks, smem, stream);
  return launch_nt<2, 4>(a, tc, ts, blocks, smem, stream);
}

}  // namespace fl
