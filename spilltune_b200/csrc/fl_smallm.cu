// Small-M frozen projection (M <= 16 tokens: decode-like steps):
//
//   Y[m, n] = sum_g scale[n, g] * sum_{k in g} X[m, k] * L[code[n, k]]  +  sum_j Ts[m, j] * Blora[n, j]
//
// the same product as fl_fwd with each 128-wide scale group factored out of
// its dot product, so the tensor-core operand is L = bf16(lut) — exactly the
// stored code for int4-sym (c - 8), the bf16-rounded codebook for NF4 — and the
// scale multiplies the fp32 partial sum of its group.
//
// At M <= 16 every weight byte is used once: the kernel has to decode the
// packed weights as fast as a single launch can stream them (a TMA stream of a
// 30 MB projection reaches ~3.5 TB/s on B200 including the ramp).  Decode is a
// per-lane copy of a 256-entry shared-memory table mapping a payload byte to
// the bf16 pair of its two codes: two integer ops and one conflict-free 32-bit
// shared load per two weights.  (The prmt product table of fl_codebook.cuh
// costs ~21 integer ops per eight weights at the integer pipe's half rate;
// measured, table lookups for every word were faster than any mix.)
//
// Layout: a CTA owns 32*TW weight rows over the whole reduction (or one
// cluster slice of it) and, before anything else, queues TMA loads of its
// first `slots` 512-column chunks (codes with the 128-byte swizzle, plus the
// chunk's scales) into a ring of shared-memory slots.  Eight warps: warp w takes
// the 128-wide scale group w % 4 of every chunk for the TW 16-row tiles of half
// w / 4.  The MMAs are warp-level (mma.sync m16n8k16) with 16 weight rows as A
// and the tokens as the 8-wide N dimension; the chunk's activations arrive in
// the same slot (TMA, 128-byte swizzle, token rows past M zero-filled).  The reduction-split CTAs of a cluster add
// their partial sums through distributed shared memory; rank 0 adds the LoRA
// term (fp32 Blora x bf16 Ts) and writes Y.
//
// Ts = bf16(s * X . A^T) is summed here, in a fixed order, from the few FP32
// partial sums that the small-M low-rank kernel launched just before
// (fl_lora_down.cu) writes; that kernel lets this grid start while it runs
// (programmatic dependent launch), and only the final reduction waits for it.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {

int make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);

namespace sm {

constexpr int kGroups = 4;                       // 128-wide scale groups per chunk
constexpr int kChunkK = 512;                     // reduction columns per ring slot
constexpr int kTilesPerWarp = 2;                 // 16-row tiles per warp
// After the main loop the table's space holds Ts [16][65] (rows padded so the
// 16 tokens of a warp's reads fall in different banks) and Blora rows [rows][64] (fp32).
constexpr int kTsStride = 65;

// Q row slabs of 16 * TW rows per CTA, each slab's chunk split over the kGroups
// scale groups: kGroups * Q consumer warps + one TMA producer warp.  The byte
// table holds a copy per lane of every entry: entry e of lane l at
// e * kRowStride + 4 l, at the start of dynamic shared memory (a constant
// address).  Q = 2 (64 rows, two CTAs per SM): 128-byte entry rows, a lookup's
// offset a byte permute (byte << 8) | 8 l shifted right by one.  Q = 4 (128
// rows, one CTA per SM): 256-byte entry rows, so the permute (byte << 8) | 4 l
// is the offset itself; the rows' upper halves stay unused.
template <int Q>
struct Layout {
  static constexpr int kWarps = kGroups * Q;
  static constexpr int kThreads = 32 * (kWarps + 1);
  static constexpr int kRowStride = Q == 4 ? 256 : 128;
  static constexpr int kTableBytes = 256 * kRowStride;
  static constexpr int kRows = 16 * kTilesPerWarp * Q;
  static constexpr int kCtasPerSm = Q == 4 ? 1 : 2;
  static_assert(Q == 2 || Q == 4, "two or four row slabs");
  static_assert((16 * kTsStride + kRows * 64) * 4 <= kTableBytes, "epilogue staging");
};

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
  const float* parts;       // [M][64][n_parts] low-rank partial sums (rank > 0)
  int n_parts;
  float s;                  // LoRA scale
  const float* lut;         // [16]
  const float* blora;       // [N, rank]
  __nv_bfloat16* Y;         // [M, N]
  uint32_t* status;
  int M, N, K, rank;
  int split;                // CTAs of a cluster along the reduction
  int slots;                // ring depth
};

// Slot layout: codes box 0 (columns 0..255 of the chunk) [rows][128 B],
// codes box 1 (256..511), eight activation boxes (64 columns each)
// [8 NT tokens][128 B], all with the 128-byte swizzle, then scales [rows][4 fp32].
__host__ __device__ constexpr int x_box_bytes(int nt) { return 8 * nt * 128; }
__host__ __device__ constexpr int slot_bytes(int rows, int nt) {
  return rows * 128 * 2 + 8 * x_box_bytes(nt) + rows * 16;
}
__host__ __device__ constexpr int slot_stride(int rows, int nt) { return (slot_bytes(rows, nt) + 1023) / 1024 * 1024; }
// Dynamic shared memory: [Q = 4: the byte table] | ring | full and empty mbarriers +
// abort word.  After the main loop the ring's space holds the partial sums
// [group][rows][16].  With Q = 2 the byte table is a static shared array.
__host__ __device__ constexpr int smem_bytes(int rows, int nt, int slots) {
  return 1024 + slots * slot_stride(rows, nt) + 2 * slots * 8 + 16;
}
template <int Q>
__host__ __device__ constexpr int dyn_smem_bytes(int nt, int slots) {
  return Layout<Q>::kTableBytes + smem_bytes(Layout<Q>::kRows, nt, slots);
}
__host__ __device__ constexpr int red_bytes(int rows) { return kGroups * rows * 16 * 4; }

// NT: 8-token tiles, 1 (M <= 8) or 2 (M <= 16).  TW: 16-row tiles per warp,
// unrolled so the MMA chains of different tiles interleave; with one tile and
// one token tile the k-steps alternate between two partial sums (PS = 2).
// Q: row slabs (Layout above).
template <int NT, int TW, int Q>
__global__ void __launch_bounds__(Layout<Q>::kThreads, Layout<Q>::kCtasPerSm)
    smallm_kernel(const __grid_constant__ CUtensorMap tm_codes,   // [N, K/2] u8, box {128, rows}, 128B swizzle
                  const __grid_constant__ CUtensorMap tm_x,       // [M, K] bf16, box {64, 8 NT}, 128B swizzle
                  const __grid_constant__ CUtensorMap tm_scales,  // [N, K/128] fp32, box {4, rows}
                  const Args args) {
  extern __shared__ uint8_t smem_raw[];
  using L = Layout<Q>;
  constexpr int kWarps = L::kWarps;
  constexpr int kThreads = L::kThreads;
  uint8_t* table = smem_raw;
  const uintptr_t ring0 = reinterpret_cast<uintptr_t>(smem_raw) + L::kTableBytes;
  uint8_t* smem = reinterpret_cast<uint8_t*>((ring0 + 1023) & ~uintptr_t(1023));
  constexpr int PS = TW * NT <= 1 ? 2 : 1;
  constexpr int rows = L::kRows;
  constexpr int sbytes = slot_stride(rows, NT);
  constexpr int kXOff = rows * 256;                    // activation boxes within a slot
  constexpr int kSOff = kXOff + 8 * x_box_bytes(NT);   // scales within a slot
  uint8_t* ring = smem;                                                    // slots x sbytes
  float* red = reinterpret_cast<float*>(ring);                             // [group][rows][16], after the loop
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + args.slots * sbytes);  // [slots]: TMA bytes landed
  uint64_t* empty = full + args.slots;                                      // [slots]: every consumer warp done
  volatile uint32_t* abort_word = reinterpret_cast<volatile uint32_t*>(empty + args.slots);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c4 = lane & 3;
  // MMA row g of a 16-row tile holds weight row pg (and g + 8 row pg + 8): the
  // two rows of an 8-lane shared-memory phase (g = 2i, 2i + 1) are then four
  // rows apart, so their code chunks fall in opposite halves of the 128-byte
  // swizzle and the 16-byte loads are conflict-free.  The scales and the
  // partial sums use the same map.
  const int pg = (g >> 1) | ((g & 1) << 2);
  const int grp = warp & (kGroups - 1);  // scale group of every chunk
  const int half = warp / kGroups;       // row slab: tiles [half * TW, half * TW + TW) of the CTA
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
    for (int i = 0; i < args.slots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWarps);
    }
    *abort_word = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_codes);
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_scales);
  }
  auto issue = [&](int k) {  // chunk c_begin + k into slot k % slots (thread 0)
    const int sl = k % args.slots;
    uint8_t* dst = ring + sl * sbytes;
    const int c = chunk_of(k);
    mbar_arrive_expect_tx(&full[sl], slot_bytes(rows, NT));
    tma_load_2d(dst, &tm_codes, c * (kChunkK / 2), n0, &full[sl]);
    tma_load_2d(dst + rows * 128, &tm_codes, c * (kChunkK / 2) + 128, n0, &full[sl]);
#pragma unroll
    for (int b = 0; b < 8; ++b) tma_load_2d(dst + kXOff + b * x_box_bytes(NT), &tm_x, c * kChunkK + 64 * b, 0, &full[sl]);
    tma_load_2d(dst + kSOff, &tm_scales, c * 4, n0, &full[sl]);
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < args.slots && i < n_ch; ++i) issue(i);
  // Per-lane byte table: entry e of lane l at table + kRowStride e + 4 l holds
  // the bf16 pair {lut[e & 15], lut[e >> 4]}.  Warp w builds entries
  // [E w, E w + E), E = 256 / kWarps, then writes them, one copy per lane.
  if (warp < kWarps) {
    constexpr int E = 256 / kWarps;
    const float mine = __ldg(args.lut + (lane & 15));
    const int e = E * warp + (lane % E);
    const uint32_t packed =
        pack_bf16x2(__shfl_sync(0xffffffffu, mine, e & 15), __shfl_sync(0xffffffffu, mine, e >> 4));
    uint32_t* tw = reinterpret_cast<uint32_t*>(table + E * warp * L::kRowStride) + lane;
#pragma unroll 8
    for (int j = 0; j < E; ++j) tw[j * (L::kRowStride / 4)] = __shfl_sync(0xffffffffu, packed, j);
  }
  __syncthreads();
  // Byte b of payload word w -> the pair of elements 2b, 2b + 1, at entry
  // byte * kRowStride + lane * 4.
  const uint32_t tab0 = smem_u32(table);
  // Permute result bytes {x.b0, w.b_i, 0, 0} = (byte_i << 8) | x.
  const uint32_t lanex = static_cast<uint32_t>(lane) * (Q == 4 ? 4 : 8);
  auto decode = [&](uint32_t w, uint32_t* out) {
    if constexpr (Q == 4) {
      // 256-byte rows: (byte << 8) | 4 lane is the offset itself.
      out[0] = lds_u32(tab0 + __byte_perm(w, lanex, 0x5504u));
      out[1] = lds_u32(tab0 + __byte_perm(w, lanex, 0x5514u));
      out[2] = lds_u32(tab0 + __byte_perm(w, lanex, 0x5524u));
      out[3] = lds_u32(tab0 + __byte_perm(w, lanex, 0x5534u));
    } else {
      // 128-byte rows: ((byte << 8) | 8 lane) >> 1.
      out[0] = lds_u32(tab0 + (__byte_perm(w, lanex, 0x5504u) >> 1));
      out[1] = lds_u32(tab0 + (__byte_perm(w, lanex, 0x5514u) >> 1));
      out[2] = lds_u32(tab0 + (__byte_perm(w, lanex, 0x5524u) >> 1));
      out[3] = lds_u32(tab0 + (__byte_perm(w, lanex, 0x5534u) >> 1));
    }
  };

  float acc[TW][NT][4];
#pragma unroll
  for (int t = 0; t < TW; ++t)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[t][nt][0] = acc[t][nt][1] = acc[t][nt][2] = acc[t][nt][3] = 0.f;

  // X of this warp's group for tokens 8 nt + g: chunk columns 128 grp + 32 c4 + 8 w + [0, 8)
  // sit in activation box 2 grp + c4 / 2, 16-byte chunk (4 (c4 % 2) + w) ^ g of the token's row.
  const int xbox = kXOff + (2 * grp + (c4 >> 1)) * x_box_bytes(NT) + g * 128;

  // Consumer warps: wait for a slot, decode + MMA this warp's group of its
  // tiles, release the slot; the producer warp refills each slot once all
  // eight consumers released it (no CTA-wide barrier per chunk).
  bool ok = true;
  if (warp == kWarps) {
    if (lane == 0) {
      int k = args.slots;
      for (; k < n_ch; ++k) {
        const int sl = k % args.slots;
        if (!mbar_wait(&empty[sl], ((k / args.slots) - 1) & 1, abort_word, args.status, kStatusTimeoutEmpty)) break;
        fence_proxy_async_smem();  // the consumers' generic reads before the async-proxy refill
        issue(k);
      }
      // Never leave the CTA with bulk copies still landing in its shared memory.
      const int issued = k < n_ch ? k : n_ch;
      for (int i = issued > args.slots ? issued - args.slots : 0; i < issued; ++i) {
        uint32_t dummy = 0;
        mbar_wait(&full[i % args.slots], (i / args.slots) & 1, &dummy, args.status, kStatusTimeoutDrain);
      }
    }
  } else {
  for (int k = 0; k < n_ch && ok; ++k) {
    const int sl = k % args.slots;
    if (!mbar_wait_warp(&full[sl], (k / args.slots) & 1, abort_word, args.status, kStatusTimeoutFull)) {
      ok = false;
      break;
    }
    {
      const uint8_t* slot = ring + sl * sbytes;
      const uint8_t* cbox = slot + (grp >> 1) * rows * 128;  // this warp's group sits in box grp/2
      const int j = (grp & 1) * 4 + c4;                       // 16-byte chunk of the row in that box
      const float* scl = reinterpret_cast<const float*>(slot + kSOff);
      uint4 q[TW][2];
#pragma unroll
      for (int t = 0; t < TW; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = 16 * (half * TW + t) + pg + 8 * h;
          q[t][h] = *reinterpret_cast<const uint4*>(cbox + r * 128 + ((j ^ (r & 7)) << 4));
        }
      float part[PS][TW][NT][4];
#pragma unroll
      for (int p = 0; p < PS; ++p)
#pragma unroll
        for (int t = 0; t < TW; ++t)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) part[p][t][nt][0] = part[p][t][nt][1] = part[p][t][nt][2] = part[p][t][nt][3] = 0.f;
      // Payload word w of the thread's 16 bytes holds columns 32c4 + 8w + [0, 8);
      // MMA k-step kk = 2w + s uses its pairs 2s (columns +4s+{0,1}) and 2s+1 (+{2,3}).
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint4 xq[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          xq[nt] = *reinterpret_cast<const uint4*>(slot + xbox + nt * 8 * 128 + (((4 * (c4 & 1) + w) ^ g) << 4));
#pragma unroll
        for (int t = 0; t < TW; ++t) {
          uint32_t e0[4], e1[4];  // rows g and g + 8
          decode(word4(q[t][0], w), e0);
          decode(word4(q[t][1], w), e1);
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            const int kk = 2 * w + sub;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint32_t b0 = sub ? xq[nt].z : xq[nt].x, b1 = sub ? xq[nt].w : xq[nt].y;
              mma16816(part[kk % PS][t][nt], e0[2 * sub], e1[2 * sub], e0[2 * sub + 1], e1[2 * sub + 1], b0, b1);
            }
          }
        }
      }
#pragma unroll
      for (int t = 0; t < TW; ++t) {
        const int r0 = 16 * (half * TW + t) + pg, r1 = r0 + 8;
        const float s0 = scl[r0 * 4 + grp], s1 = scl[r1 * 4 + grp];
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
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[sl]);
  }
  }

  // ------------------------------------------------------------ reductions
  // Warp partials -> red[group][row][token] in the ring's space, once every
  // copy into the ring has landed (the consumers waited for each chunk; the
  // producer drained what an abort left in flight): accumulator element i of
  // tile t: row 16 (half TW + t) + pg + 8*(i >> 1), token 8*nt + 2*c4 + (i & 1).
  __syncthreads();
  if (warp < kWarps)
#pragma unroll
  for (int t = 0; t < TW; ++t) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        red[(grp * rows + 16 * (half * TW + t) + pg + 8 * (i >> 1)) * 16 + 8 * nt + 2 * c4 + (i & 1)] = acc[t][nt][i];
  }
  __syncthreads();
  // Sum the four groups into red[0] (tokens past 8*NT stay unused).
  for (int idx = threadIdx.x; idx < rows * 16; idx += kThreads)
    red[idx] = red[idx] + red[rows * 16 + idx] + red[2 * rows * 16 + idx] + red[3 * rows * 16 + idx];
  if (split > 1) {
    cluster_sync();
  } else {
    __syncthreads();
  }
  if (kslice == 0) {
    // The table's space now holds Ts and this tile's Blora rows.
    float* ts = reinterpret_cast<float*>(table);
    float* bl = ts + 16 * kTsStride;
    if (args.rank > 0) {
      // Blora rows first: they do not depend on the low-rank kernel.
#pragma unroll 4
      for (int idx = threadIdx.x; idx < rows * args.rank; idx += kThreads) {
        const int r = idx / args.rank, jj = idx % args.rank;
        bl[r * 64 + jj] = n0 + r < args.N ? __ldg(args.blora + static_cast<size_t>(n0) * args.rank + idx) : 0.f;
      }
      griddep_wait();
      // Ts[m][j] = bf16(s * sum of the partials in order).
      const int n_cl = args.n_parts;
      for (int o = threadIdx.x; o < args.M * args.rank; o += kThreads) {
        const int m = o / args.rank, jj = o % args.rank;
        const float* src = args.parts + (static_cast<size_t>(m) * 64 + jj) * n_cl;
        float v = 0.f;
#pragma unroll 4
        for (int c = 0; c < n_cl; ++c) v += __ldg(src + c);
        ts[m * kTsStride + jj] = __bfloat162float(__float2bfloat16_rn(args.s * v));
      }
      __syncthreads();
    }
    const uint32_t red_local = smem_u32(red);
    for (int idx = threadIdx.x; idx < rows * 16; idx += kThreads) {
      const int lr = idx >> 4, tok = idx & 15;
      const int n = n0 + lr;
      if (n < args.N && tok < args.M) {
        float v = red[idx];
        for (int p = 1; p < split; ++p)
          v += __uint_as_float(ld_shared_cluster_u32(mapa_shared(red_local, static_cast<uint32_t>(p)) + idx * 4));
        if (args.rank > 0) {
          const float* tr = ts + tok * kTsStride;
          const float* br = bl + lr * 64;
          for (int jj = 0; jj < args.rank; ++jj) v = fmaf(tr[jj], br[jj], v);
        }
        args.Y[static_cast<size_t>(tok) * args.N + n] = __float2bfloat16_rn(v);
      }
    }
  }
  if (split > 1) cluster_sync();  // peers' partials stay valid until rank 0 has read them
}

// Split of the reduction across a cluster while the grid still fits in one
// wave of `slots` resident CTAs and every CTA keeps two 512-wide chunks.
static int cluster_split(int blocks, int chunks, int slots) {
  int split = 1;
  while (split < 8 && blocks * split * 2 <= slots && chunks >= 2 * split) split *= 2;
  return split;
}

// CTAs of smallm_kernel<NT, TW, Q> resident per SM with `slots` ring slots (sets
// the kernel's shared-memory limit once per device and ring depth).
template <int NT, int TW, int Q>
static int resident_per_sm(int slots, int* per_sm) {
  static int cache[64][9] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || slots < 1 || slots > 8)
    return set_error(FL_ERR_CUDA, "small-M: no current device");
  if (!cache[dev][slots]) {
    const int smem = dyn_smem_bytes<Q>(NT, slots);
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&smallm_kernel<NT, TW, Q>),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int n = 0;
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, smallm_kernel<NT, TW, Q>, Layout<Q>::kThreads, smem);
    if (e != cudaSuccess || n < 1) return set_error(FL_ERR_CUDA, "small-M occupancy query failed");
    cache[dev][slots] = n;
  }
  *per_sm = cache[dev][slots];
  return FL_OK;
}

template <int NT, int TW, int Q>
static int launch_tw(Args a, const void* codes, const float* scales, bool pdl, cudaStream_t stream) {
  using L = Layout<Q>;
  constexpr int rows = L::kRows;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    sms = 148;
  // Ring depth: the most slots that still fit next to the table at the
  // occupancy the registers allow.
  constexpr int want_ctas = L::kCtasPerSm;
  int slots = 2;
  while (slots < 6 && want_ctas * (smem_bytes(rows, NT, slots + 1) + L::kTableBytes + 1024) <= 233472) ++slots;
  if (want_ctas * (smem_bytes(rows, NT, slots) + L::kTableBytes + 1024) > 233472 ||
      red_bytes(rows) > slots * slot_stride(rows, NT))
    return set_error(FL_ERR_CUDA, "small-M: shared-memory plan does not fit");
  int per_sm = 1;
  int rc = resident_per_sm<NT, TW, Q>(slots, &per_sm);
  if (rc) return rc;
  const int blocks = (a.N + rows - 1) / rows;
  // Too few row blocks for one full wave: split the reduction across a cluster.
  const int chunks = a.K / kChunkK;
  const int split = cluster_split(blocks, chunks, per_sm * sms);
  a.split = split;
  a.slots = slots;
  CUtensorMap tc, tx, ts;
  rc = make_tensor_map_2d(&tc, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.K / 2, a.N, a.K / 2, 128, rows,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tensor_map_2d(&tx, a.X, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.K, a.M, static_cast<uint64_t>(a.K) * 2, 64,
                          8 * NT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tensor_map_2d(&ts, scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.K / 128, a.N,
                          static_cast<uint64_t>(a.K / 128) * 4, 4, rows, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks * split);
  cfg.blockDim = dim3(L::kThreads);
  cfg.dynamicSmemBytes = dyn_smem_bytes<Q>(NT, slots);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  cudaError_t le = cudaLaunchKernelEx(&cfg, smallm_kernel<NT, TW, Q>, tc, tx, ts, a);
  if (le != cudaSuccess) return set_error(FL_ERR_CUDA, "small-M launch: %s", cudaGetErrorString(le));
  return FL_OK;
}

}  // namespace sm

int launch_smallm_fwd(const void* X, const float* lora_parts, float s, const uint8_t* codes, const float* scales,
                      const float* lut, const float* lora, int rank, void* Y, int M, int N, int K, cudaStream_t stream,
                      int layout) {
  using namespace sm;
  if (M < 1 || M > 16) return set_error(FL_ERR_ARG, "small-M path needs 1 <= M <= 16");
  if (K % kChunkK != 0) return set_error(FL_ERR_ARG, "small-M path needs K %% 512 == 0");
  if (layout != 0) return set_error(FL_ERR_UNSUPPORTED, "small-M path: group-128 records only");
  Args a;
  a.X = static_cast<const __nv_bfloat16*>(X);
  a.parts = lora_parts;
  a.n_parts = K / (128 * lora_parts_per_cluster(K));
  a.s = s;
  a.lut = lut;
  a.blora = lora;
  a.Y = static_cast<__nv_bfloat16*>(Y);
  int dev = 0;
  cudaGetDevice(&dev);
  a.status = status_word(dev);
  a.M = M;
  a.N = N;
  a.K = K;
  a.rank = rank;
  a.split = 1;
  a.slots = 2;
  // With a LoRA term the preceding launch produced Ts: start while it runs.
  const bool pdl = rank > 0;
  // One token tile (M <= 8): 128-row CTAs with the byte-permute table (Q = 4)
  // when each CTA still streams at least four chunks.  Measured against Q = 2
  // (back-to-back calls over cold copies): 14336x4096 18.5 -> 17.7 us,
  // 4096x14336 22.3 -> 21.8 us, 6144x4096 14.3 -> 14.0 us; with two chunks per
  // CTA (4096x4096, 1024x4096) and with two token tiles Q = 4 was 2-6% slower.
  if (M <= 8) {
    int sms = 148;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 148;
    const int chunks = K / kChunkK;
    const bool long_ctas = chunks / cluster_split((N + 127) / 128, chunks, sms) >= 4;
    return long_ctas ? launch_tw<1, kTilesPerWarp, 4>(a, codes, scales, pdl, stream)
                     : launch_tw<1, kTilesPerWarp, 2>(a, codes, scales, pdl, stream);
  }
  return launch_tw<2, kTilesPerWarp, 2>(a, codes, scales, pdl, stream);
}

}  // namespace fl
