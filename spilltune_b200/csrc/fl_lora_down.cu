// lora_down: the low-rank projection of the LoRA branch,
//
//   Lo[m, j] = bf16( s * sum_r P[m, r] * Q(j, r) ),  j < rank (<= 64), zero for rank <= j < 64,
//
// forward: P = X, Q = Alora (the reference's F.linear(x.float(), A),
// finetune/lora.py:219) -> Ts;  backward: P = dY, Q = Blora^T (the VJP factor
// dY.float() @ B, training/recompute.py:102-105) -> Us.
//
// HBM-bound: it streams P once, so the kernel is built for memory-level
// parallelism.
//  * A prepass turns the FP32 factor into a bf16 hi/lo pair (hi + lo equals
//    the FP32 value to ~16 mantissa bits) laid out in the order the warp MMA
//    fragments read it, [plane][unit u of 64 r][j][c][16]: a warp's fragment
//    loads are 1 KiB contiguous and stay in L1 for the CTA's other warps.
//  * A producer warp streams each 64-wide unit of the CTA's 128 rows into a
//    ring of kStages shared-memory stages: one TMA box {64 columns, 128 rows}
//    (128-byte swizzle) plus the unit's slice of the converted factor (one
//    contiguous bulk copy per plane).  Four consumer warps (32 rows each)
//    read both from shared memory, so the factor never competes for the
//    small L1 left next to the stages.  Rows past the segment's end (another
//    expert's rows in a grouped launch) are read but never stored: every
//    output row is its own dot product.
//    The reduction index inside a unit is permuted so that one thread's 16
//    consecutive r feed four m16n8k16 steps: physical r = 16c + 4i + {0..3}
//    plays logical k = {2c, 2c+1, 2c+8, 2c+9} of step i, for both operands.
//  * The CTAs of a cluster split the reduction; their partial sums meet in
//    distributed shared memory, each CTA finishing 1/split of the rows.
//  * The backward's Us pass (P = dY, rank <= 16) also sums dB = dY^T . Ts: per
//    unit each consumer warp takes 16 of its 64 columns over all 128 rows,
//    reading the dY tile transposed (ldmatrix) with Ts fragments kept in
//    registers, and adds the result into dB with global reductions, so dY
//    crosses HBM once for both.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {

int make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);

namespace ld {

constexpr int kWarps = 4;                       // consumer warps
constexpr int kRowsPerWarp = 32;
constexpr int kRows = kWarps * kRowsPerWarp;    // 128 rows per CTA
constexpr int kThreads = 32 * (kWarps + 1);     // + one producer warp
constexpr int kMaxSplit = 8;
constexpr int kStages = 4;
constexpr int kChunks = 8;                      // 16-byte chunks per thread per unit
constexpr int kXBytes = kRows * 128;            // 16 KiB: 128 rows x 64 bf16

template <int NQ>
struct Cfg {
  static constexpr int kQPlane = NQ * 128;      // one plane of a unit's converted factor
  static constexpr int kStage = kXBytes + 2 * kQPlane;
  static constexpr int kSmem = 1024 /*align*/ + kStages * kStage + 2 * kStages * 8 /*mbarriers*/ +
                               kRows * (NQ + 1) * 4;
};

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Prepass: qc[e][plane][u][j][c][16] (bf16) from Q(j, r) = q[e*q_es + j*q_sj + r*q_sr],
// one thread per (e, j, 8 consecutive r); then, after expert e's two planes,
// one 32-bit mask per 64-wide unit u: bit n set when some Q(j, r) with
// 8n <= j < 8n + 8, r in the unit, is nonzero (one warp per unit).  A
// block-diagonal factor (the LoRA branches of several projections over one
// input, stacked) leaves most 8-column groups of a unit zero; lora_down skips
// their MMAs.  qc_es: elements from one expert's block to the next.
__global__ void prep_kernel(const float* __restrict__ q, int64_t q_sj, int64_t q_sr, int64_t q_es, int rank, int R,
                            int nq, int experts, __nv_bfloat16* __restrict__ qc, int64_t qc_es) {
  // lora_down follows at once (programmatic dependent launch) and starts
  // streaming its activations; it waits for this grid before reading qc.
  griddep_launch_dependents();
  const int r8s = R / 8;
  const int64_t total = static_cast<int64_t>(experts) * nq * r8s;
  const int64_t plane = static_cast<int64_t>(nq) * R;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r8 = static_cast<int>(idx % r8s);
    const int j = static_cast<int>((idx / r8s) % nq);
    const int e = static_cast<int>(idx / (static_cast<int64_t>(r8s) * nq));
    const int r0 = r8 * 8;
    float v[8];
    if (j < rank) {
      const float* src = q + e * q_es + j * q_sj + static_cast<int64_t>(r0) * q_sr;
      if (q_sr == 1 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(src));
        const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = __ldg(src + t * q_sr);
      }
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = 0.f;
    }
    uint32_t h[4], l[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      h[t] = pack_bf16x2(v[2 * t], v[2 * t + 1]);
      const float h0 = __uint_as_float(h[t] << 16), h1 = __uint_as_float(h[t] & 0xFFFF0000u);
      l[t] = pack_bf16x2(v[2 * t] - h0, v[2 * t + 1] - h1);
    }
    const int u = r0 >> 6, c = (r0 & 63) >> 4, w = r0 & 15;
    const int64_t off = ((static_cast<int64_t>(u) * nq + j) * 4 + c) * 16 + w;
    __nv_bfloat16* base = qc + static_cast<int64_t>(e) * qc_es;
    *reinterpret_cast<uint4*>(base + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(base + plane + off) = make_uint4(l[0], l[1], l[2], l[3]);
  }
  // Unit masks: warp `wid` takes unit u of expert e; lane l looks at r = 64u + l
  // and 64u + 32 + l for every j < rank.
  const int units = R / 64;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t wid = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
       wid < static_cast<int64_t>(experts) * units; wid += warps) {
    const int u = static_cast<int>(wid % units);
    const int e = static_cast<int>(wid / units);
    const float* src = q + e * q_es + static_cast<int64_t>(64 * u + lane) * q_sr;
    uint32_t mask = 0;
    for (int n = 0; n < nq / 8; ++n) {
      // The group's 16 loads go out together (unrolled, predicated), so a unit
      // costs one memory round trip per group instead of one per column.
      float v[16];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int j = 8 * n + i;
        v[2 * i] = j < rank ? __ldg(src + j * q_sj) : 0.f;
        v[2 * i + 1] = j < rank ? __ldg(src + j * q_sj + 32 * q_sr) : 0.f;
      }
      bool any = false;
#pragma unroll
      for (int i = 0; i < 16; ++i) any |= v[i] != 0.f;
      if (__any_sync(0xffffffffu, any)) mask |= 1u << n;
    }
    if (lane == 0) reinterpret_cast<uint32_t*>(qc + static_cast<int64_t>(e) * qc_es + 2 * plane)[u] = mask;
  }
  // Launched as a dependent itself (the second factor of a backward): finish
  // no earlier than the launch before, so completion stays ordered.
  griddep_wait();
}

__device__ __forceinline__ uint32_t word(const uint4& a, const uint4& b, int w) {
  const uint4& q = w < 4 ? a : b;
  const int k = w & 3;
  return k == 0 ? q.x : k == 1 ? q.y : k == 2 ? q.z : q.w;
}

// kGrad (NQ == 16 only): the launch also adds grad[r, j] += sum_m P[m, r] *
// Lo2[m, j] (j < rank) for every r of its units, from the P tiles already in
// shared memory: with P = dY and Lo2 = Ts that is dB = dY^T . Ts of the
// reference's LoRA backward (training/recompute.py:102-127), so the backward
// streams dY once for Us and dB instead of twice.
template <int NQ, bool kGrad = false>
__global__ void __launch_bounds__(kThreads)
    lora_down_kernel(const __grid_constant__ CUtensorMap tm_p,  // P [M, R] bf16, box {64, 128}, 128B swizzle
                     int M, int R, const __nv_bfloat16* __restrict__ qc, int64_t qc_es, int rank, float s,
                     __nv_bfloat16* __restrict__ out, int split, const int4* __restrict__ tiles,
                     const int* __restrict__ tile_count, uint32_t* status,
                     const __nv_bfloat16* __restrict__ lo2,  // kGrad: [M, 64] bf16 (Ts), zero past the rank
                     float* __restrict__ grad,               // kGrad: [R, rank] fp32 per expert, added into
                     int64_t grad_es) {                      // kGrad, grouped: floats from one expert's grad to the next
  static_assert(!kGrad || NQ == 16, "the gradient pass keeps Lo2 fragments for rank <= 16 in registers");
  using C = Cfg<NQ>;
  constexpr int NT = NQ / 8;  // n-tiles of 8 rank columns
  // A launch of the stream that may overlap this one (programmatic dependent
  // launch, the small-M backward) waits for its completion before reading out.
  griddep_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * C::kStage);
  uint64_t* empty = full + kStages;
  auto red = reinterpret_cast<float (*)[NQ + 1]>(smem + kStages * C::kStage + 2 * kStages * 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int kslice = split > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int blk = blockIdx.x / split;
  int m0 = blk * kRows, m_end = M;
  if (tiles != nullptr) {
    // MoE: one <= 128-row tile of one expert's segment (every CTA of the
    // cluster reads the same entry, so they leave together).
    if (blk >= *tile_count) return;
    const int4 t = tiles[blk];
    m0 = t.y;
    m_end = min(t.z, M);
    qc += t.x * qc_es;
    if constexpr (kGrad) grad += t.x * grad_es;
  }
  const int64_t plane = static_cast<int64_t>(NQ) * R;
  const int units = R / 64;
  // Per 64-wide unit: which 8-column groups of the factor are nonzero (the prepass).
  const uint32_t* umask = reinterpret_cast<const uint32_t*>(qc + 2 * plane);
  const int u0 = kslice * units / split;
  const int u1 = (kslice + 1) * units / split;
  const int n_units = u1 - u0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  uint32_t abort_local = 0;
  volatile uint32_t* abort_word = &abort_local;

  float acc[2][NT][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int n = 0; n < NT; ++n) acc[t][n][0] = acc[t][n][1] = acc[t][n][2] = acc[t][n][3] = 0.f;

  if (warp == kWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_p);
      // The activations of the first ring's worth of units go out at once; the
      // converted factor is the previous launch's output (programmatic
      // dependent launch of the prepass): wait for that grid before reading it.
      const int pre = n_units < kStages ? n_units : kStages;
      for (int k = 0; k < pre; ++k) {
        mbar_arrive_expect_tx(&full[k], C::kStage);
        tma_load_2d(smem + k * C::kStage, &tm_p, (u0 + k) * 64, m0, &full[k]);
      }
      griddep_wait();
      int issued = 0;
      for (int k = 0; k < n_units; ++k) {
        const int st = k % kStages;
        const int u = u0 + k;
        uint8_t* stage = smem + st * C::kStage;
        const __nv_bfloat16* qsrc = qc + static_cast<int64_t>(u) * NQ * 64;
        if (k >= pre) {
          if (!mbar_wait_short(&empty[st], ((k / kStages) - 1) & 1, abort_word, status, kStatusTimeoutEmpty)) break;
          mbar_arrive_expect_tx(&full[st], C::kStage);
          tma_load_2d(stage, &tm_p, u * 64, m0, &full[st]);
        }
        bulk_load(stage + kXBytes, qsrc, C::kQPlane, &full[st]);
        bulk_load(stage + kXBytes + C::kQPlane, qsrc + plane, C::kQPlane, &full[st]);
        ++issued;
      }
      for (int i = issued > kStages ? issued - kStages : 0; i < issued; ++i) {
        uint32_t dummy = 0;
        mbar_wait_short(&full[i % kStages], (i / kStages) & 1, &dummy, status, kStatusTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    // The unit masks are the prepass grid's output, like qc: wait for that grid
    // (the producer does the same before loading qc).
    griddep_wait();
    // kGrad: B fragments of Lo2 for the CTA's 128 rows (8 k-steps of 16 rows x
    // two 8-column tiles), lane (g, c) holding rows 2c, 2c + 1 (+8) of column g.
    uint32_t lo2f[kGrad ? 8 : 1][2][2];
    if constexpr (kGrad) {
      const uint16_t* l2 = reinterpret_cast<const uint16_t*>(lo2);
      auto at = [&](int row, int col) -> uint32_t {
        const int m = m0 + row;
        return m < m_end ? static_cast<uint32_t>(l2[static_cast<size_t>(m) * 64 + col]) : 0u;
      };
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
#pragma unroll
        for (int rt = 0; rt < 2; ++rt) {
          const int col = 8 * rt + g, r0 = 16 * kk + 2 * c;
          lo2f[kk][rt][0] = at(r0, col) | (at(r0 + 1, col) << 16);
          lo2f[kk][rt][1] = at(r0 + 8, col) | (at(r0 + 9, col) << 16);
        }
    }
    for (int k = 0; k < n_units; ++k) {
      const int st = k % kStages;
      const uint32_t um = umask[u0 + k];
      if (!mbar_wait_short_warp(&full[st], (k / kStages) & 1, abort_word, status, kStatusTimeoutFull)) break;
      const uint8_t* stage = smem + st * C::kStage;
      // Thread (g, c) needs chunk 2c + e of rows 32w + 16t + 8h + g; under the
      // 128-byte swizzle chunk j of row r sits at position j ^ (r % 8).
      uint4 x[kChunks];
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int r = warp * kRowsPerWarp + 16 * t + 8 * h + g;
            x[(t * 2 + h) * 2 + e] =
                *reinterpret_cast<const uint4*>(stage + r * 128 + (((2 * c + e) ^ (r & 7)) << 4));
          }
      const uint8_t* qb = stage + kXBytes + ((g * 4 + c) * 16) * 2;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        if (((um >> n) & 1u) == 0) continue;  // this unit's 8 factor columns are all zero
        const uint4* hp = reinterpret_cast<const uint4*>(qb + n * 8 * 64 * 2);
        const uint4* lp = reinterpret_cast<const uint4*>(qb + C::kQPlane + n * 8 * 64 * 2);
        const uint4 h0 = hp[0], h1 = hp[1];
        const uint4 l0 = lp[0], l1 = lp[1];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t bh0 = word(h0, h1, 2 * i), bh1 = word(h0, h1, 2 * i + 1);
          const uint32_t bl0 = word(l0, l1, 2 * i), bl1 = word(l0, l1, 2 * i + 1);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            // rows g (h = 0) and g + 8 (h = 1): chunk (t*2 + h)*2 + e
            const uint32_t a0 = word(x[(t * 2 + 0) * 2], x[(t * 2 + 0) * 2 + 1], 2 * i);
            const uint32_t a1 = word(x[(t * 2 + 1) * 2], x[(t * 2 + 1) * 2 + 1], 2 * i);
            const uint32_t a2 = word(x[(t * 2 + 0) * 2], x[(t * 2 + 0) * 2 + 1], 2 * i + 1);
            const uint32_t a3 = word(x[(t * 2 + 1) * 2], x[(t * 2 + 1) * 2 + 1], 2 * i + 1);
            mma_16816(acc[t][n], a0, a1, a2, a3, bh0, bh1);
            mma_16816(acc[t][n], a0, a1, a2, a3, bl0, bl1);
          }
        }
      }
      if constexpr (kGrad) {
        // grad rows r = 64u + 16 warp + [0, 16) over the CTA's 128 rows of P: A = P^T
        // (16 r x 16 rows of P per k-step, transposed out of the swizzled tile by
        // ldmatrix: matrix i covers r-half i & 1 and row-half i >> 1), B = Lo2.
        float gacc[2][4];
#pragma unroll
        for (int rt = 0; rt < 2; ++rt) gacc[rt][0] = gacc[rt][1] = gacc[rt][2] = gacc[rt][3] = 0.f;
        const uint32_t stage_s = smem_u32(stage);
        const int mi = lane >> 3;
        const int chunk = 2 * warp + (mi & 1);  // 16-byte chunk (8 r) of the 128-byte row
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int row = 16 * kk + 8 * (mi >> 1) + (lane & 7);
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4_trans(stage_s + row * 128 + ((chunk ^ (row & 7)) << 4), a0, a1, a2, a3);
#pragma unroll
          for (int rt = 0; rt < 2; ++rt) mma_16816(gacc[rt], a0, a1, a2, a3, lo2f[kk][rt][0], lo2f[kk][rt][1]);
        }
        const int rbase = (u0 + k) * 64 + 16 * warp + g;
#pragma unroll
        for (int rt = 0; rt < 2; ++rt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = rbase + 8 * (i >> 1), j = 8 * rt + 2 * c + (i & 1);
            if (j < rank && r < R) atomicAdd(grad + static_cast<size_t>(r) * rank + j, gacc[rt][i]);
          }
      }
      // The stage's values are in registers: hand it back to the producer.
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  }

  // Partial sums -> shared memory (rows of this CTA, NQ columns).
  if (warp < kWarps) {
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int r = warp * kRowsPerWarp + 16 * t + g;
      red[r][8 * n + 2 * c] = acc[t][n][0];
      red[r][8 * n + 2 * c + 1] = acc[t][n][1];
      red[r + 8][8 * n + 2 * c] = acc[t][n][2];
      red[r + 8][8 * n + 2 * c + 1] = acc[t][n][3];
    }
  }
  if (split > 1) {
    cluster_sync();
  } else {
    __syncthreads();
  }
  // This CTA finishes rows [r_begin, r_end) of the 128: sum the split
  // partials, scale, round, write 64 bf16 per row (zero past the rank).
  const int r_begin = kslice * kRows / split;
  const int r_end = (kslice + 1) * kRows / split;
  const uint32_t red_local = smem_u32(&red[0][0]);
  for (int idx = threadIdx.x; idx < (r_end - r_begin) * 8; idx += kThreads) {
    const int r = r_begin + idx / 8, q8 = idx % 8;  // output columns 8*q8 .. +7
    const int m = m0 + r;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 0.f;
    if (8 * q8 < NQ) {
      if (split > 1) {
        for (int p = 0; p < split; ++p) {
          const uint32_t base =
              mapa_shared(red_local, static_cast<uint32_t>(p)) + static_cast<uint32_t>((r * (NQ + 1) + 8 * q8) * 4);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] += __uint_as_float(ld_shared_cluster_u32(base + 4 * e));
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = red[r][8 * q8 + e];
      }
    }
    if (m < m_end) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j0 = 8 * q8 + 2 * e;
        w[e] = pack_bf16x2(j0 < rank ? s * v[2 * e] : 0.f, j0 + 1 < rank ? s * v[2 * e + 1] : 0.f);
      }
      *reinterpret_cast<uint4*>(out + static_cast<size_t>(m) * 64 + 8 * q8) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  // Peers read this CTA's partials: stay until every CTA of the cluster is done.
  if (split > 1) cluster_sync();
}

// CTAs of lora_down_kernel<NQ, kGrad> resident on the current device at once
// (sets the kernel's shared-memory limit once per device); 0 on failure.
template <int NQ, bool kGrad>
static int resident_slots() {
  constexpr int kSmem = Cfg<NQ>::kSmem;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  static int slots[64] = {0};
  if (!slots[dev]) {
    int sms = 0, per_sm = 0;
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&lora_down_kernel<NQ, kGrad>),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lora_down_kernel<NQ, kGrad>, kThreads, kSmem);
    if (e != cudaSuccess || per_sm < 1) return 0;
    slots[dev] = sms * per_sm;
  }
  return slots[dev];
}

// Split the reduction across a cluster while the grid still fits in one
// wave of resident CTAs and every slice keeps at least two 64-wide units.
static int cluster_split(int blocks, int R, int slots) {
  int split = 1;
  while (split < kMaxSplit && blocks * split * 2 <= slots && (R / 64) >= 4 * split) split *= 2;
  return split;
}

template <int NQ, bool kGrad = false>
static int launch_nq(const void* P, int M, int R, const __nv_bfloat16* qc, int64_t qc_es, int rank, float s,
                     void* out, cudaStream_t stream, const int4* tiles, const int* tile_count, int max_tiles,
                     const void* lo2 = nullptr, float* grad = nullptr, int64_t grad_es = 0) {
  const int blocks = tiles ? max_tiles : (M + kRows - 1) / kRows;
  if (blocks < 1) return FL_OK;
  constexpr int kSmem = Cfg<NQ>::kSmem;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return set_error(FL_ERR_CUDA, "lora_down: no current device");
  const int slots = resident_slots<NQ, kGrad>();
  if (slots < 1) return set_error(FL_ERR_CUDA, "lora_down: occupancy query failed");
  const int split = cluster_split(blocks, R, slots);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks * split);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  // A programmatic dependent of the prepass that converted qc (the launch
  // just before it): the producer waits for that grid before reading qc.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  CUtensorMap tm;
  int rc = make_tensor_map_2d(&tm, P, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, R, M, static_cast<uint64_t>(R) * 2, 64,
                              kRows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cudaError_t le = cudaLaunchKernelEx(&cfg, lora_down_kernel<NQ, kGrad>, tm, M, R, qc, qc_es, rank, s,
                                      static_cast<__nv_bfloat16*>(out), split, tiles, tile_count, status_word(dev),
                                      static_cast<const __nv_bfloat16*>(lo2), grad, grad_es);
  if (le != cudaSuccess) return set_error(FL_ERR_CUDA, "lora_down launch: %s", cudaGetErrorString(le));
  return FL_OK;
}

}  // namespace ld

// Small-M form (at most 16 rows of P, rows of Q contiguous along r): the work
// is a few MFLOP, so the kernel is built for latency.  Block y takes the ranks
// j = 8y + w (one per warp w); a warp's lanes take four consecutive r of
// every 128-wide piece of the CTA's slice of the reduction and keep one exact
// FP32 sum per row of P.  The CTAs of a cluster split the reduction; CTA 0
// adds their sums in rank order.  The kernel first lets the next launch of the
// stream start (programmatic dependent launch): the small-M frozen projection
// streams its weights meanwhile and reads Lo only once this grid completed.
namespace lds {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxRows = 16;
constexpr int kMaxSplit = 8;

__global__ void __launch_bounds__(kThreads)
    lora_down_small_kernel(const __nv_bfloat16* __restrict__ P, int M, int R, const float* __restrict__ q,
                           int64_t q_sj, int rank, float s, __nv_bfloat16* __restrict__ out, int split) {
  griddep_launch_dependents();
  __shared__ float part[kWarps * kMaxRows];  // [warp][m]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cr = split > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int pieces = R / 128;
  const int p0 = cr * pieces / split, p1 = (cr + 1) * pieces / split;
  const int j = blockIdx.y * kWarps + warp;
  float acc[kMaxRows];
#pragma unroll
  for (int m = 0; m < kMaxRows; ++m) acc[m] = 0.f;
  if (j < rank) {
    const float* qrow = q + j * q_sj;
    for (int p = p0; p < p1; ++p) {
      const int r = p * 128 + lane * 4;
      const float4 qv = __ldg(reinterpret_cast<const float4*>(qrow + r));
#pragma unroll
      for (int m = 0; m < kMaxRows; ++m) {
        if (m < M) {
          const uint2 xv = __ldg(reinterpret_cast<const uint2*>(P + static_cast<size_t>(m) * R + r));
          acc[m] = fmaf(__uint_as_float(xv.x << 16), qv.x, acc[m]);
          acc[m] = fmaf(__uint_as_float(xv.x & 0xFFFF0000u), qv.y, acc[m]);
          acc[m] = fmaf(__uint_as_float(xv.y << 16), qv.z, acc[m]);
          acc[m] = fmaf(__uint_as_float(xv.y & 0xFFFF0000u), qv.w, acc[m]);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < kMaxRows; ++m)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
  if (lane < kMaxRows) {
    float v = 0.f;
#pragma unroll
    for (int m = 0; m < kMaxRows; ++m) v = lane == m ? acc[m] : v;
    part[warp * kMaxRows + lane] = v;
  }
  __syncthreads();
  if (split > 1) cluster_sync();
  if (cr == 0) {
    const uint32_t local = smem_u32(part);
    // This block's ranks; block 0 also writes the zero columns [rank, 64).
    const int j0 = blockIdx.y * kWarps;
    const int j_end = blockIdx.y == 0 ? 64 : min(j0 + kWarps, rank);
    const int width = j_end - j0;
    for (int idx = threadIdx.x; idx < M * width; idx += kThreads) {
      const int m = idx / width, jj = j0 + idx % width;
      float v = 0.f;
      if (jj < rank && jj < j0 + kWarps) {
        const int off = (jj - j0) * kMaxRows + m;
        for (int c = 0; c < split; ++c)
          v += c == 0 ? part[off]
                      : __uint_as_float(ld_shared_cluster_u32(mapa_shared(local, static_cast<uint32_t>(c)) +
                                                              static_cast<uint32_t>(off) * 4));
        v *= s;
      }
      if (jj >= rank || jj < j0 + kWarps) out[static_cast<size_t>(m) * 64 + jj] = __float2bfloat16_rn(v);
    }
  }
  if (split > 1) cluster_sync();  // peers' sums stay valid until CTA 0 has read them
}

static int launch(const void* P, int M, int R, const float* q, int64_t q_sj, int rank, float s, void* out,
                  cudaStream_t stream) {
  int split = 1;
  while (split < kMaxSplit && (R / 128) >= 2 * split) split *= 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(split, (rank + kWarps - 1) / kWarps);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t le = cudaLaunchKernelEx(&cfg, lora_down_small_kernel, static_cast<const __nv_bfloat16*>(P), M, R, q,
                                      q_sj, rank, s, static_cast<__nv_bfloat16*>(out), split);
  if (le != cudaSuccess) return set_error(FL_ERR_CUDA, "lora_down (small M) launch: %s", cudaGetErrorString(le));
  return FL_OK;
}


// One reduction of a lora_parts launch: P [M, R] bf16, Q(j, r) = q[j * q_sj + r * q_sr].
struct PartsJob {
  const __nv_bfloat16* P;
  const float* q;
  int64_t q_sj, q_sr;
  float* parts;
  int R;
};

// Partial form for the small-M forward and backward: CTA p takes the 128-wide piece p of the
// reduction (exact FP32 sums in shared memory); the clusters of lora_parts_per_cluster(R0, R1)
// CTAs add their pieces in rank order through distributed shared memory, and
// cluster c writes parts[m][j][c] (j < rank; the partials of one output
// contiguous) for the consumer to add in order.  One piece per CTA keeps every
// CTA to a single round of loads, so the kernel finishes early even while the
// frozen projection that follows (programmatic dependent launch) streams its
// weights on the same SMs.
// One launch runs one or two reductions: blocks [0, R0/128) take job 0, the
// rest job 1 (clusters never straddle: csize divides both piece counts).
__global__ void __launch_bounds__(kThreads)
    lora_parts_kernel(const PartsJob j0, const PartsJob j1, int M, int rank, int csize) {
  griddep_launch_dependents();
  __shared__ float mine[kMaxRows * 64];  // [m][j] of this CTA's piece
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pieces0 = j0.R / 128;
  const bool second = static_cast<int>(blockIdx.x) >= pieces0;
  const __nv_bfloat16* P = second ? j1.P : j0.P;
  const float* q = second ? j1.q : j0.q;
  const int64_t q_sj = second ? j1.q_sj : j0.q_sj, q_sr = second ? j1.q_sr : j0.q_sr;
  float* parts = second ? j1.parts : j0.parts;
  const int R = second ? j1.R : j0.R;
  const int blk = second ? static_cast<int>(blockIdx.x) - pieces0 : static_cast<int>(blockIdx.x);
  const int r = blk * 128 + lane * 4;
  uint2 xv[kMaxRows];
#pragma unroll
  for (int m = 0; m < kMaxRows; ++m)
    xv[m] = m < M ? __ldg(reinterpret_cast<const uint2*>(P + static_cast<size_t>(m) * R + r)) : make_uint2(0, 0);
  for (int j = warp; j < rank; j += kWarps) {
    float4 qv;
    if (q_sr == 1) {
      qv = __ldg(reinterpret_cast<const float4*>(q + j * q_sj + r));
    } else {
      const float* qj = q + j * q_sj + r * q_sr;
      qv = make_float4(__ldg(qj), __ldg(qj + q_sr), __ldg(qj + 2 * q_sr), __ldg(qj + 3 * q_sr));
    }
    float acc[kMaxRows];
#pragma unroll
    for (int m = 0; m < kMaxRows; ++m) {
      float a = __uint_as_float(xv[m].x << 16) * qv.x;
      a = fmaf(__uint_as_float(xv[m].x & 0xFFFF0000u), qv.y, a);
      a = fmaf(__uint_as_float(xv[m].y << 16), qv.z, a);
      acc[m] = fmaf(__uint_as_float(xv[m].y & 0xFFFF0000u), qv.w, a);
    }
#pragma unroll
    for (int m = 0; m < kMaxRows; ++m)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
    float v = 0.f;
#pragma unroll
    for (int m = 0; m < kMaxRows; ++m) v = lane == m ? acc[m] : v;
    if (lane < kMaxRows) mine[lane * 64 + j] = v;
  }
  cluster_sync();
  const int crank = static_cast<int>(cluster_ctarank());
  if (crank == 0) {
    const int n_cl = (R / 128) / csize;
    const int cl = blk / csize;
    const uint32_t local = smem_u32(mine);
    for (int idx = threadIdx.x; idx < M * rank; idx += kThreads) {
      const int m = idx / rank, j = idx % rank;
      const uint32_t off = static_cast<uint32_t>(m * 64 + j) * 4;
      float v = mine[m * 64 + j];
      for (int c = 1; c < csize; ++c)
        v += __uint_as_float(ld_shared_cluster_u32(mapa_shared(local, static_cast<uint32_t>(c)) + off));
      parts[(static_cast<size_t>(m) * 64 + j) * n_cl + cl] = v;
    }
  }
  cluster_sync();  // peers' sums stay valid until rank 0 has read them
}

}  // namespace lds

static bool parts_job_ok(const void* P, int R, const float* q, int64_t q_sj, int64_t q_sr, const float* parts) {
  if (R % 128 != 0 || R <= 0) return false;
  if ((reinterpret_cast<uintptr_t>(P) | reinterpret_cast<uintptr_t>(parts)) & 15u) return false;
  if (q_sr == 1 && ((reinterpret_cast<uintptr_t>(q) & 15u) || q_sj % 4 != 0)) return false;
  return true;
}

int lora_parts_per_cluster(int R0, int R1) {
  auto one = [](int R) {
    const int pieces = R / 128;
    return pieces % 8 == 0 ? 8 : pieces % 4 == 0 ? 4 : pieces % 2 == 0 ? 2 : 1;
  };
  const int a = one(R0);
  if (R1 <= 0) return a;
  const int b = one(R1);
  return a < b ? a : b;
}

int launch_lora_parts2(const void* P0, int R0, const float* q0, int64_t q0_sj, int64_t q0_sr, float* parts0,
                       const void* P1, int R1, const float* q1, int64_t q1_sj, int64_t q1_sr, float* parts1, int M,
                       int rank, cudaStream_t stream) {
  if (M < 1 || M > lds::kMaxRows || rank < 1 || rank > 64)
    return set_error(FL_ERR_ARG, "lora_parts: needs 1 <= M <= 16, 1 <= rank <= 64");
  if (!parts_job_ok(P0, R0, q0, q0_sj, q0_sr, parts0) || (R1 > 0 && !parts_job_ok(P1, R1, q1, q1_sj, q1_sr, parts1)))
    return set_error(FL_ERR_ARG, "lora_parts: needs R %% 128 == 0 and 16-byte aligned activations, factor, partials");
  const int csize = lora_parts_per_cluster(R0, R1);
  lds::PartsJob j0{static_cast<const __nv_bfloat16*>(P0), q0, q0_sj, q0_sr, parts0, R0};
  lds::PartsJob j1{static_cast<const __nv_bfloat16*>(P1), q1, q1_sj, q1_sr, parts1, R1 > 0 ? R1 : 0};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(R0 / 128 + (R1 > 0 ? R1 / 128 : 0));
  cfg.blockDim = dim3(lds::kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, lds::lora_parts_kernel, j0, j1, M, rank, csize);
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "lora_parts launch: %s", cudaGetErrorString(e));
  return FL_OK;
}

int launch_lora_parts(const void* P, int M, int R, const float* q, int64_t q_sj, int64_t q_sr, int rank,
                      float* parts, cudaStream_t stream) {
  return launch_lora_parts2(P, R, q, q_sj, q_sr, parts, nullptr, 0, nullptr, 0, 1, nullptr, M, rank, stream);
}

int lora_nq(int rank) { return rank <= 16 ? 16 : rank <= 32 ? 32 : 64; }

// Per expert: the hi and lo planes (2 x nq x R bf16) and the unit masks (R / 64
// uint32, padded to 16 bytes).
size_t lora_factor_bytes(int64_t R, int rank) {
  return 4u * static_cast<size_t>(lora_nq(rank)) * R + static_cast<size_t>((R / 64 * 4 + 15) / 16 * 16);
}

int launch_lora_down(const void* P, int M, int R, const float* q, int64_t q_sj, int64_t q_sr, int rank, float s,
                     void* out64, void* qc_scratch, cudaStream_t stream, const int4* tiles, const int* tile_count,
                     int max_tiles, int64_t q_expert_stride, int experts, bool pdl, const void* lo2, float* grad,
                     bool* grad_done) {
  if (grad_done) *grad_done = false;
  if (R % 64 != 0) return set_error(FL_ERR_ARG, "lora_down: reduction dim %d not a multiple of 64", R);
  if (rank < 1 || rank > 64) return set_error(FL_ERR_ARG, "lora_down: rank %d outside [1, 64]", rank);
  if ((reinterpret_cast<uintptr_t>(P) | reinterpret_cast<uintptr_t>(out64) |
       reinterpret_cast<uintptr_t>(qc_scratch)) & 15u)
    return set_error(FL_ERR_ARG, "lora_down: activations, output and scratch must be 16-byte aligned");
  // The small-M kernel takes 128-wide pieces of the reduction; the tiled
  // kernel 64-wide units (any R % 64 == 0).
  if (tiles == nullptr && M <= lds::kMaxRows && R % 128 == 0 && q_sr == 1 && q_sj % 4 == 0 &&
      (reinterpret_cast<uintptr_t>(q) & 15u) == 0)
    return lds::launch(P, M, R, q, q_sj, rank, s, out64, stream);
  const int nq = lora_nq(rank);
  auto qc = static_cast<__nv_bfloat16*>(qc_scratch);
  {
    const int64_t total = static_cast<int64_t>(experts) * nq * (R / 8);
    const int threads = 256;
    // Enough threads for the conversion and one warp per unit for the masks.
    const int64_t items = total > static_cast<int64_t>(experts) * (R / 64) * 32 ? total
                                                                                : static_cast<int64_t>(experts) * (R / 64) * 32;
    const int64_t want = (items + threads - 1) / threads;
    const int grid = static_cast<int>(want < 4096 ? want : 4096);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const int64_t qc_es = static_cast<int64_t>(lora_factor_bytes(R, rank) / 2);
    cudaError_t e = cudaLaunchKernelEx(&cfg, ld::prep_kernel, q, q_sj, q_sr, q_expert_stride, rank, R, nq, experts, qc,
                                       qc_es);
    if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "lora_down prepass: %s", cudaGetErrorString(e));
  }
  const int64_t qc_es = static_cast<int64_t>(lora_factor_bytes(R, rank) / 2);
  if (nq == 16 && grad != nullptr && lo2 != nullptr) {
    if ((reinterpret_cast<uintptr_t>(lo2) & 15u) != 0)
      return set_error(FL_ERR_ARG, "lora_down: Lo2 must be 16-byte aligned");
    // Grouped launches: expert e's gradient sits one factor's size after e - 1's.
    const int rc = ld::launch_nq<16, true>(P, M, R, qc, qc_es, rank, s, out64, stream, tiles, tile_count, max_tiles,
                                           lo2, grad, q_expert_stride);
    if (rc == FL_OK && grad_done) *grad_done = true;
    return rc;
  }
  if (nq == 16) return ld::launch_nq<16>(P, M, R, qc, qc_es, rank, s, out64, stream, tiles, tile_count, max_tiles);
  if (nq == 32) return ld::launch_nq<32>(P, M, R, qc, qc_es, rank, s, out64, stream, tiles, tile_count, max_tiles);
  return ld::launch_nq<64>(P, M, R, qc, qc_es, rank, s, out64, stream, tiles, tile_count, max_tiles);
}

int lora_down_ctas(int M, int R, int rank) {
  using namespace ld;
  if (M <= lds::kMaxRows || rank < 1 || rank > 64 || R % 64 != 0) return 0;
  const int blocks = (M + kRows - 1) / kRows;
  const int nq = lora_nq(rank);
  const int slots = nq == 16 ? resident_slots<16, false>() : nq == 32 ? resident_slots<32, false>()
                                                                       : resident_slots<64, false>();
  return blocks * cluster_split(blocks, R, slots > 0 ? slots : 148);
}

}  // namespace fl
