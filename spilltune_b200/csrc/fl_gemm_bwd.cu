// Backward of the frozen projection (weight-gradient free), fused with the
// 4-bit decode and the LoRA branch:
//
//   dX[M,K] = dY[M,N] . W[N,K] + Us[M,r] . Alora[r,K],   Us = bf16(s * dY . Blora)
//
// the autograd VJP the reference takes for F.linear(x, W) + the FP32 LoRA
// F.linears inside StreamingBlockFunction.backward
// (ram_vram_finetune/training/recompute.py:85-127, finetune/lora.py:218-220).
//
// Mapping (CTA pair, tcgen05 cta_group::2, both operands in shared memory):
//   * MMA M = 256 tokens (128 per CTA; the A operand is the dY tile, TMA-loaded
//     K-major with the 128-byte swizzle), N = 256 columns k of W (128 per CTA;
//     the B operand), K = the reduction over W rows n in 64-wide stages.
//   * B = W[n0:n0+64, kb:kb+128] is decoded in its stored orientation: a thread
//     owns one row n and 64 consecutive k, builds that row's 16-entry product
//     table once (bit-identical to decode_into), looks codes up four at a time
//     with prmt and writes 128-byte rows of the MN-major 128-byte-swizzled
//     operand layout.  No transpose is needed.
//   * Every accumulator lane is one token row of dX, so the epilogue writes 64
//     contiguous bytes per thread per 32-column chunk.
//   * The extra LoRA stage uses A = the Us tile, B = bf16(Alora[0:64, k]).
// Persistent CTA pairs over a static tile list with two TMEM accumulators
// (512 columns), in one of two forms (Cfg below):
//   * 256-token tiles: tile t+1 accumulates while tile t drains; 6 stages,
//     three decode groups (448 threads per CTA);
//   * 512-token tiles (dense launches with many tokens): every decoded W stage
//     feeds both accumulators (tokens m0.. and m0+256..), half the decode per
//     FLOP; the next tile's MMAs wait for the drain; two dY tiles per stage
//     leave room for 4 stages and two decode groups (320 threads per CTA).
// Warp roles: warp 0 TMA producer, warp 1 TMEM owner (both CTAs) + MMA issuer
// (leader), then the groups of four decode warps that take turns on stages
// and drain the previous tile's accumulator(s) after their first stage pair
// of the next one.  Barriers as in fl_gemm.cu, with
// accum/acc_empty per accumulator.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_codebook.cuh"
#include "fl_ptx.cuh"

namespace fl {
namespace bwd {

constexpr int kTokHalf = 128;              // tokens per CTA (A rows)
constexpr int kColHalf = 128;              // W columns k per CTA (B rows)
constexpr int kStageN = 64;                // reduction rows n per stage
constexpr int kGroupM = 4;                 // token tiles per band: a band's pairs fit in one wave, so each dY slab is read once
constexpr int kAccCols = 256;              // fp32 accumulator columns (pair N)
constexpr int kTmemCols = 2 * kAccCols;    // two accumulators: tile t+1 accumulates while tile t drains
constexpr int kABytes = kTokHalf * kStageN * 2;   // 16 KiB dY (or Us) tile
constexpr int kBBytes = kColHalf * kStageN * 2;   // 16 KiB decoded W tile
constexpr int kQBytes = kStageN * kColHalf / 2;   // 4 KiB packed codes
constexpr uint32_t kBLbo = 1024;           // MN-direction atom stride (64 k per atom)
constexpr uint32_t kBSbo = 2048;           // K-direction 8-row group stride

template <int S>
struct __align__(16) BarriersT {
  uint64_t full[S];
  uint64_t afull[S];
  uint64_t empty[S];
  uint64_t accum[2];        // accumulator b holds a finished tile (one phase per use)
  uint64_t acc_empty[2];    // leader: both CTAs' epilogue warps drained accumulator b
  uint32_t tmem_base;
  uint32_t abort_word;
  alignas(16) float lut[16];
};

// kW token tiles of 256 per pair tile.  kW = 1: the two TMEM accumulators
// alternate between tiles (tile t+1 accumulates while tile t drains).  kW = 2
// (dense launches with many tokens): each decoded W stage feeds both
// accumulators, tokens [m0, m0 + 256) and [m0 + 256, m0 + 512), halving the
// decode per FLOP; the next tile waits for the drain, and the two dY tiles per
// stage leave room for 4 stages and 2 decode groups.
template <int kW>
struct Cfg {
  static constexpr int kStages = kW == 2 ? 4 : 6;
  static constexpr int kGroups = kW == 2 ? 2 : 3;  // decode warp groups
  static constexpr int kThreads = 64 + 128 * kGroups;
  static constexpr int kEpiWarps = 4 * kGroups;
  using Bars = BarriersT<kStages>;
  static constexpr int kSmemBytes = 1024 + kStages * (kW * kABytes + kBBytes + kQBytes) + static_cast<int>(sizeof(Bars));
  // A decode group's consecutive stages are at most 2 * kGroups apart; at most
  // kStages keeps its parity waits on a ring slot within one phase.
  static_assert(2 * kGroups <= kStages, "decode-group rotation longer than the stage ring");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct Args {
  const float* scales;
  const float* lut;
  const float* alora;   // [r, K] (grouped: [E, r, K])
  __nv_bfloat16* out;   // dX [M, K]
  uint32_t* status;
  int M, N, K, rank;
  const int4* tiles;    // MoE: {expert, first row, end row, column tile}; null for one weight
  const int* tile_count;
  // Dense launches with a split reduction: ksplit > 1 slices of N / ksplit,
  // FP32 sums to part[kpart][M][K] (dX is then formed by the split reduce).
  float* part;
  int ksplit;
  // 512-token launches: tiles [0, dense_full) are full 512-token tiles; the
  // last round's remaining wide tiles follow as two 256-token halves each
  // (one accumulator), so the last round costs about half.
  int dense_full;
};

// Byte offset of 16-byte chunk j (k = 8j..8j+7 within the CTA's 64-k half
// `khalf`) of reduction row r in the MN-major swizzled B tile.
__device__ __forceinline__ uint32_t b_offset(int r, int khalf, int j) {
  return khalf * kBLbo + (r >> 3) * kBSbo + (r & 7) * 128 + ((j ^ (r & 7)) << 4);
}

struct Tile {
  int expert, m0, m_end, k_tile, kpart, half;  // half: a 256-token tile of a 512-token launch
};
// Tile t: grouped launches read the list; dense ones walk bands of kGroupM
// token tiles x all column tiles, so a band's dY slab is read by pairs that
// run together.
__device__ __forceinline__ Tile tile_at(const Args& args, int t, int num_k, int num_m, int tok_tile) {
  Tile r;
  r.half = 0;
  if (args.tiles != nullptr) {
    const int4 v = args.tiles[t];
    r.expert = v.x;
    r.m0 = v.y;
    r.m_end = v.z;
    r.k_tile = v.w;
    r.kpart = 0;
  } else {
    int sub = 0;
    if (t >= args.dense_full) {  // (512-token launches) half h of wide tile dense_full + j
      const int j = t - args.dense_full;
      sub = j & 1;
      t = args.dense_full + (j >> 1);
      r.half = 1;
    }
    // The slices of one output tile are consecutive tiles (they run together).
    r.kpart = t % args.ksplit;
    t /= args.ksplit;
    const int band = t / (kGroupM * num_k);
    const int first_m = band * kGroupM;
    const int rows_in_band = min(kGroupM, num_m - first_m);
    const int local = t - band * kGroupM * num_k;
    r.expert = 0;
    r.m0 = (first_m + local % rows_in_band) * tok_tile + sub * (tok_tile / 2);
    r.m_end = args.M;
    r.k_tile = local / rows_in_band;
  }
  return r;
}

// Persistent: each CTA pair walks tiles pair, pair + P, ...; stage counters
// run on across tiles.  kW = 1: the two TMEM accumulators alternate, so the
// MMAs of the next tile overlap the drain of the previous one; kW = 2: both
// hold one 512-token tile and the next tile's MMAs wait for its drain.
template <int kLayout, int kW>
__global__ void __launch_bounds__(Cfg<kW>::kThreads, 1)
    fl_bwd_ss_kernel(const __grid_constant__ CUtensorMap tm_dy,    // dY [M, N] bf16, box {64, 128}
                     const __grid_constant__ CUtensorMap tm_us,    // Us [M, 64] bf16, box {64, 128}
                     const __grid_constant__ CUtensorMap tm_code,  // payload [E*N, K/2] u8, box {64, 64}, 64B swizzle
                     const Args args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using C = Cfg<kW>;
  constexpr int kStages = C::kStages;
  constexpr int kGroups = C::kGroups;
  constexpr int kEpiWarps = C::kEpiWarps;
  using Barriers = typename C::Bars;
  uint8_t* as = smem;                                  // kStages x kW x 16 KiB (stage s, token half h at s * kW + h)
  uint8_t* bs = as + kStages * kW * kABytes;           // kStages x 16 KiB
  uint8_t* qs = bs + kStages * kBBytes;                // kStages x 4 KiB
  Barriers* bars = reinterpret_cast<Barriers*>(qs + kStages * kQBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = args.M, N = args.N, K = args.K;
  const int groups_per_row = K / 128;
  const uint32_t crank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_k = (K + 2 * kColHalf - 1) / (2 * kColHalf);
  constexpr int kTokTile = 2 * kTokHalf * kW;   // tokens per pair tile
  const int num_m = (M + kTokTile - 1) / kTokTile;
  // 512-token launches: the last round's wide tiles as two halves each.
  const int n_dense = num_k * num_m * args.ksplit;
  const int n_tiles = args.tiles != nullptr ? *args.tile_count : 2 * n_dense - min(args.dense_full, n_dense);
  const int n_main = N / kStageN / args.ksplit;  // stages of one tile's reduction slice
  const bool has_lora = args.rank > 0;
  const int n_iter = n_main + (has_lora ? 1 : 0);
  volatile uint32_t* abort_word = &bars->abort_word;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->afull[s], 2 * 4);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->accum[b], 1);
      mbar_init(&bars->acc_empty[b], 2 * kEpiWarps);
    }
    bars->abort_word = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < 16) bars->lut[threadIdx.x] = __ldg(args.lut + threadIdx.x);
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
      tma_prefetch_desc(&tm_dy);
      tma_prefetch_desc(&tm_code);
      if (has_lora) tma_prefetch_desc(&tm_us);
      int g = 0;
      bool ok = true;
      bool us_ready = false;
      for (int t = pair; t < n_tiles && ok; t += num_pairs) {
        const Tile tile = tile_at(args, t, num_k, num_m, kTokTile);
        const int kb = tile.k_tile * 2 * kColHalf + static_cast<int>(crank) * kColHalf;
        const int mh = tile.m0 + static_cast<int>(crank) * kTokHalf;
        const int wrow0 = tile.expert * N;
        for (int it = 0; it < n_iter; ++it, ++g) {
          const int s = g % kStages;
          if (g >= kStages &&
              !mbar_wait(&bars->empty[s], ((g / kStages) - 1) & 1, abort_word, args.status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (it < n_main) {
            const int n0 = (tile.kpart * n_main + it) * kStageN;
            const int na = tile.half ? 1 : kW;  // dY tiles of this tile
            mbar_arrive_expect_tx(&bars->full[s], na * kABytes + kQBytes);
#pragma unroll
            for (int h = 0; h < kW; ++h)
              if (h < na) tma_load_2d(as + (s * kW + h) * kABytes, &tm_dy, n0, mh + h * 2 * kTokHalf, &bars->full[s]);
            tma_load_2d(qs + s * kQBytes, &tm_code, kb / 2, wrow0 + n0, &bars->full[s]);
          } else {
            // Us comes from an earlier launch of the call chain (programmatic
            // dependent launch): wait for the previous grid, whose completion
            // implies every earlier one's, before the first read.  Only then
            // may the gradient kernels that read Us and Ts launch.
            if (!us_ready) {
              griddep_wait();
              griddep_launch_dependents();
              us_ready = true;
            }
            const int na = tile.half ? 1 : kW;
            mbar_arrive_expect_tx(&bars->full[s], na * kABytes);
#pragma unroll
            for (int h = 0; h < kW; ++h)
              if (h < na) tma_load_2d(as + (s * kW + h) * kABytes, &tm_us, 0, mh + h * 2 * kTokHalf, &bars->full[s]);
          }
        }
      }
      // Finish no earlier than the previous launch (also on the abort path).
      griddep_wait();
      for (int i = g > kStages ? g - kStages : 0; i < g; ++i) {
        uint32_t dummy_abort = 0;
        mbar_wait(&bars->full[i % kStages], (i / kStages) & 1, &dummy_abort, args.status, kStatusTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    if (lane == 0 && crank == 0) {
      const uint32_t idesc = idesc_bf16_f32_bmn(2 * kTokHalf, 2 * kColHalf);
      const int lora_k_steps = (args.rank + 15) / 16;
      int g = 0, tl = 0;
      bool ok = true;
      for (int t = pair; t < n_tiles && ok; t += num_pairs, ++tl) {
        // kW = 1: accumulator b was last used by tile tl-2; kW = 2: both were
        // used by tile tl-1.  Both CTAs must have drained it.
        const int b = kW == 2 ? 0 : (tl & 1);
        const bool reused = kW == 2 ? tl >= 1 : tl >= 2;
        const uint32_t ph_empty = kW == 2 ? ((tl - 1) & 1) : (((tl >> 1) - 1) & 1);
        if (reused && !mbar_wait_cluster(&bars->acc_empty[b], ph_empty, abort_word, args.status, kStatusTimeoutAccum))
          break;
        tc_fence_after();
        const int na = tile_at(args, t, num_k, num_m, kTokTile).half ? 1 : kW;  // accumulators this tile fills
        for (int it = 0; it < n_iter; ++it, ++g) {
          const int s = g % kStages;
          const uint32_t ph = (g / kStages) & 1;
          if (!mbar_wait_cluster(&bars->afull[s], ph, abort_word, args.status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = sdesc_mnmajor_sw128(smem_u32(bs + s * kBBytes), kBLbo, kBSbo);
          const int ksteps = it < n_main ? kStageN / 16 : lora_k_steps;
#pragma unroll
          for (int h = 0; h < kW; ++h) {
            if (h >= na) break;
            const uint64_t adesc = sdesc_kmajor_sw128(smem_u32(as + (s * kW + h) * kABytes));
            const uint32_t acc = tmem_base + (kW == 2 ? h : b) * kAccCols;
            for (int kk = 0; kk < ksteps; ++kk)
              mma_ss2(acc, adesc + 2 * kk, bdesc + ((2 * kBSbo) >> 4) * kk, idesc, (it | kk) != 0 ? 1u : 0u);
          }
          tc_commit2_mc(&bars->empty[s], 0x3);
        }
        tc_commit2_mc(&bars->accum[b], 0x3);
      }
      if (tl > 0) {
        // The last commit covers every MMA this thread issued.
        uint32_t dummy_abort = 0;
        const int last = tl - 1;
        if (kW == 2)
          mbar_wait(&bars->accum[0], last & 1, &dummy_abort, args.status, kStatusTimeoutAccum);
        else
          mbar_wait(&bars->accum[last & 1], (last >> 1) & 1, &dummy_abort, args.status, kStatusTimeoutAccum);
      }
    }
  } else {
    // ------------------------------------------------------------ decode warps
    const int dw = warp - 2;
    const int grp = dw >> 2;                 // stage-pair group
    // Lanes 0-15 take 16 rows' first 64 columns, lanes 16-31 the same rows'
    // second 64: the eight lanes of a 16-byte shared-memory phase then hold eight
    // consecutive rows, whose swizzled chunks (decoded B rows, codes) fall on
    // distinct banks.
    const int r = (dw & 3) * 16 + (lane & 15);  // reduction row within the stage (0..63)
    const int khalf = lane >> 4;                // which 64 of the CTA's 128 columns
    const uint32_t afull_leader = mapa_shared(smem_u32(&bars->afull[0]), 0);
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(&bars->acc_empty[0]), 0);
    const int quarter = warp & 3;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;

    // Epilogue of the pair's tl-th tile: lane quarter q holds tokens
    // mh + 32q .. +32; each thread writes its token row's columns in 32-wide
    // chunks (64 contiguous bytes), the groups taking chunks round robin.
    auto epilogue = [&](const Tile& tile, int tl) {
      const int b = kW == 2 ? 0 : (tl & 1);
      const uint32_t ph_acc = kW == 2 ? (tl & 1) : ((tl >> 1) & 1);
      const int k0 = tile.k_tile * 2 * kColHalf;
      if (ok && mbar_wait_warp(&bars->accum[b], ph_acc, abort_word, args.status, kStatusTimeoutAccum)) {
        tc_fence_after();
#pragma unroll 1
        for (int h = 0; h < (tile.half ? 1 : kW); ++h) {
        // Token half h of the tile: accumulator h (kW = 2) or b.
        const int m = tile.m0 + h * 2 * kTokHalf + static_cast<int>(crank) * kTokHalf + quarter * 32 + lane;
        const uint32_t acc_col = static_cast<uint32_t>((kW == 2 ? h : b) * kAccCols);
#pragma unroll 1
        for (int c = 32 * grp; c < kAccCols; c += 32 * kGroups) {
          uint32_t acc[32];
          tmem_ld_32x32b_x32(tmem_base + acc_col + lane_addr + c, acc);
          tmem_wait_ld();
          const int kcol = k0 + c;
          if (args.ksplit > 1) {
            // FP32 sums of this reduction slice: 128 contiguous bytes per thread.
            if (m < tile.m_end && kcol < K) {
              float4* dst = reinterpret_cast<float4*>(args.part + (static_cast<size_t>(tile.kpart) * M + m) * K + kcol);
#pragma unroll
              for (int j = 0; j < 8; ++j)
                dst[j] = make_float4(__uint_as_float(acc[4 * j]), __uint_as_float(acc[4 * j + 1]),
                                     __uint_as_float(acc[4 * j + 2]), __uint_as_float(acc[4 * j + 3]));
            }
          } else if (m < tile.m_end && kcol < K) {
            uint4* dst = reinterpret_cast<uint4*>(args.out + static_cast<size_t>(m) * K + kcol);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint4 o;
              o.x = pack_bf16x2(__uint_as_float(acc[8 * j + 0]), __uint_as_float(acc[8 * j + 1]));
              o.y = pack_bf16x2(__uint_as_float(acc[8 * j + 2]), __uint_as_float(acc[8 * j + 3]));
              o.z = pack_bf16x2(__uint_as_float(acc[8 * j + 4]), __uint_as_float(acc[8 * j + 5]));
              o.w = pack_bf16x2(__uint_as_float(acc[8 * j + 6]), __uint_as_float(acc[8 * j + 7]));
              dst[j] = o;
            }
          }
        }
        }
        tc_fence_before();
      } else {
        ok = false;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader + b * 8);
    };

    // Per tile: the group's first stage pair, then the previous tile's
    // epilogue, then the rest; the other accumulator keeps the MMAs busy.
    int g0 = 0;
    int tl = 0;
    Tile prev{};
    const int pairs_per_tile = (n_iter + 1) / 2;  // the last one a single stage when n_iter is odd
    for (int tt = pair; tt < n_tiles; tt += num_pairs, g0 += n_iter, ++tl) {
      const Tile tile = tile_at(args, tt, num_k, num_m, kTokTile);
      const int kb = tile.k_tile * 2 * kColHalf + static_cast<int>(crank) * kColHalf;
      const int wrow0 = tile.expert * N;
      const float* alora = args.alora + static_cast<size_t>(tile.expert) * args.rank * K;
      const bool tile_valid = kb < K;
      const int nbase = tile.kpart * n_main * kStageN;  // first reduction row of the tile's slice
      // Layout 0: the CTA's 128 columns share one 128-group scale; layout 1:
      // each thread's 64 columns are one 64-block.
      constexpr bool kBlock64 = kLayout == kLayoutNf4Dq64;
      const int spr = kBlock64 ? 2 * groups_per_row : groups_per_row;
      const int gsc = tile_valid ? (kBlock64 ? kb / 64 + khalf : kb / 128) : 0;
      // The row's scales for the group's next stage pair (stages 2g, 2g+1,
      // 2g+2*kGroups, ...) are loaded when the current pair starts: a whole
      // rotation of the groups ahead, so the gather has landed when used.
      auto load_scale = [&](int it) {
        return (tile_valid && it < n_main)
                   ? __ldg(args.scales + static_cast<size_t>(wrow0 + nbase + it * kStageN + r) * spr + gsc)
                   : 0.0f;
      };
      // The groups take the stage pairs of the CTA pair's whole stage sequence
      // in turn (tile tl starts a new pair, number tl * pairs_per_tile), not
      // afresh per tile: consecutive stages of one group are then never more
      // than 2 * kGroups == kStages apart, so a group never waits on a ring
      // slot whose barrier is two phases behind (the parity wait would pass).
      const int first = (grp - (tl * pairs_per_tile) % kGroups + kGroups) % kGroups;
      const int pit0 = 2 * first;
      float next0 = load_scale(pit0), next1 = load_scale(pit0 + 1);
      for (int pit = pit0; pit < n_iter || (pit == pit0 && tl > 0); pit += 2 * kGroups) {
        const float pair_scale[2] = {next0, next1};
        next0 = load_scale(pit + 2 * kGroups);
        next1 = load_scale(pit + 2 * kGroups + 1);
        if (pit < n_iter && ok) {
          for (int it = pit; it < pit + 2 && it < n_iter; ++it) {
            const int gi = g0 + it;
            const int s = gi % kStages;
            const uint32_t ph = (gi / kStages) & 1;
            if (gi >= kStages &&
                !mbar_wait_warp(&bars->empty[s], ((gi / kStages) - 1) & 1, abort_word, args.status,
                                kStatusTimeoutEmpty)) {
              ok = false;
              break;
            }
            uint32_t v[32];
            const float scale = pair_scale[it - pit];
            if (it < n_main) {
              const ProductTable table = make_table(bars->lut, scale);
              if (!mbar_wait_warp(&bars->full[s], ph, abort_word, args.status, kStatusTimeoutFull)) {
                ok = false;
                break;
              }
              // Row r's 16-byte chunk c sits at chunk c ^ ((r >> 1) & 3) (64-byte swizzle).
              const uint8_t* qrow = qs + s * kQBytes + r * 64;
              const uint32_t sw = (r >> 1) & 3;
              const uint4 q0 = *reinterpret_cast<const uint4*>(qrow + (((2 * khalf) ^ sw) << 4));
              const uint4 q1 = *reinterpret_cast<const uint4*>(qrow + (((2 * khalf + 1) ^ sw) << 4));
              lookup8_l<kLayout>(table, q0.x, v + 0);
              lookup8_l<kLayout>(table, q0.y, v + 4);
              lookup8_l<kLayout>(table, q0.z, v + 8);
              lookup8_l<kLayout>(table, q0.w, v + 12);
              lookup8_l<kLayout>(table, q1.x, v + 16);
              lookup8_l<kLayout>(table, q1.y, v + 20);
              lookup8_l<kLayout>(table, q1.z, v + 24);
              lookup8_l<kLayout>(table, q1.w, v + 28);
            } else {
              // LoRA stage: row r of B is bf16(Alora[r, kb + 64*khalf .. +64]), zero past the rank.
              if (!mbar_wait_warp(&bars->full[s], ph, abort_word, args.status, kStatusTimeoutFull)) {
                ok = false;
                break;
              }
              const bool live = tile_valid && tile.kpart == 0 && r < args.rank;  // a split sums it once
              const float* src = alora + static_cast<size_t>(live ? r : 0) * K + kb + 64 * khalf;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                float2 a = make_float2(0.f, 0.f);
                if (live) a = __ldg(reinterpret_cast<const float2*>(src) + j);
                v[j] = pack_bf16x2(a.x, a.y);
              }
            }
            uint8_t* dst = bs + s * kBBytes;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<uint4*>(dst + b_offset(r, khalf, j)) =
                  make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(afull_leader + s * 8);
          }
          ok = __all_sync(0xffffffffu, ok) != 0;
        }
        if (pit == pit0 && tl > 0) epilogue(prev, tl - 1);
      }
      prev = tile;
    }
    if (tl > 0) epilogue(prev, tl - 1);
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

}  // namespace bwd
}  // namespace fl

// ------------------------------------------------------------------ host side
#include <cuda_runtime.h>

#include "fl_host.h"

namespace fl {

int make_tensor_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);

// Persistent CTA pairs, no more than can be resident at once (each tile:
// 256 tokens x 256 columns of dX).
int launch_bwd_gemm(const void* dy, const void* us, const uint8_t* codes, const float* scales, const float* lut,
                    const float* alora, int rank, void* dx, int M, int N, int K, uint32_t* status,
                    cudaStream_t stream, const int4* tiles, const int* tile_count, int experts, int max_tiles,
                    int layout, bool pdl, float* part, int ksplit, bool grouped_wide) {
  using namespace bwd;
  if (layout != kLayoutG128 && layout != kLayoutNf4Dq64) return set_error(FL_ERR_ARG, "bwd gemm: unknown layout");
  if (layout != kLayoutG128 && tiles) return set_error(FL_ERR_UNSUPPORTED, "grouped launches use layout 0");
  if ((K * 2) % 16 != 0 || N % kStageN != 0 || K % 128 != 0)
    return set_error(FL_ERR_ARG, "bwd gemm: needs N %% 64 == 0 and K %% 128 == 0");
  if (ksplit < 1 || (ksplit > 1 && (tiles || !part || (N / kStageN) % ksplit != 0)))
    return set_error(FL_ERR_ARG, "bwd gemm: invalid reduction split %d", ksplit);
  CUtensorMap tm_dy, tm_us, tm_code;
  int rc = make_tensor_map_2d(&tm_dy, dy, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, N, M, static_cast<uint64_t>(N) * 2, 64,
                              kTokHalf, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (rank > 0) {
    rc = make_tensor_map_2d(&tm_us, us, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 64, M, 128, 64, kTokHalf,
                            CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    tm_us = tm_dy;
  }
  rc = make_tensor_map_2d(&tm_code, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, static_cast<uint64_t>(N) * experts,
                          K / 2, kColHalf / 2, kStageN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  Args a;
  a.scales = scales;
  a.lut = lut;
  a.alora = alora;
  a.out = static_cast<__nv_bfloat16*>(dx);
  a.status = status;
  a.M = M;
  a.N = N;
  a.K = K;
  a.rank = rank;
  a.tiles = tiles;
  a.tile_count = tile_count;
  a.part = part;
  a.ksplit = ksplit;
  // 512-token pair tiles (each decoded W stage feeds both accumulators) for
  // dense launches without a reduction split, with a reduction over N >=
  // kBwdWideMinN (measured: 16-32 stages of 64 rows gained nothing or lost 1%,
  // the next tile waiting for the drain; 64 and more stages gained 8-16%), when
  // the pairs' rounds of wide tiles, each costing 1.62 rounds of 256-token
  // tiles (measured 1.53-1.62 at 8192 tokens), beat the rounds of 256-token
  // tiles; for grouped launches exactly when the caller planned 512-row tiles.
  const int num_k = (K + 2 * kColHalf - 1) / (2 * kColHalf);
  const int64_t P = device_pairs();
  const int64_t narrow_rounds = (static_cast<int64_t>(num_k) * ((M + 2 * kTokHalf - 1) / (2 * kTokHalf)) + P - 1) / P;
  const int64_t wide_rounds = (static_cast<int64_t>(num_k) * ((M + 4 * kTokHalf - 1) / (4 * kTokHalf)) + P - 1) / P;
  const bool wide = tiles ? grouped_wide
                          : (ksplit == 1 && N >= kBwdWideMinN && 162 * wide_rounds < 100 * narrow_rounds);
  const int tok_tile = (wide ? 4 : 2) * kTokHalf;
  const int tiles_max = tiles ? max_tiles : num_k * ((M + tok_tile - 1) / tok_tile) * ksplit;
  const void* kfn;
  if (layout == kLayoutG128)
    kfn = wide ? reinterpret_cast<const void*>(&fl_bwd_ss_kernel<kLayoutG128, 2>)
               : reinterpret_cast<const void*>(&fl_bwd_ss_kernel<kLayoutG128, 1>);
  else
    kfn = wide ? reinterpret_cast<const void*>(&fl_bwd_ss_kernel<kLayoutNf4Dq64, 2>)
               : reinterpret_cast<const void*>(&fl_bwd_ss_kernel<kLayoutNf4Dq64, 1>);
  const int threads = wide ? Cfg<2>::kThreads : Cfg<1>::kThreads;
  const int smem = wide ? Cfg<2>::kSmemBytes : Cfg<1>::kSmemBytes;
  int pairs = 0;
  if ((rc = resident_pairs(kfn, threads, smem, &pairs))) return rc;
  // 512-token launches whose last round would hold at most half a round of
  // wide tiles run those tiles as two 256-token halves each: the pairs that
  // take one finish in about 0.6 of a wide tile instead of a whole one.
  int n_tiles = tiles_max;
  a.dense_full = tiles ? 0 : tiles_max;
  if (!tiles && wide && pairs > 0) {
    const int full = (tiles_max / pairs) * pairs, rem = tiles_max - full;
    if (full > 0 && rem > 0 && 2 * rem <= pairs) {
      a.dense_full = full;
      n_tiles = full + 2 * rem;
    }
  }
  if (pairs > n_tiles) pairs = n_tiles;
  if (pairs < 1) return FL_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl && rank > 0 ? 2 : 1;
  cudaError_t le;
  if (layout == kLayoutG128)
    le = wide ? cudaLaunchKernelEx(&cfg, fl_bwd_ss_kernel<kLayoutG128, 2>, tm_dy, tm_us, tm_code, a)
              : cudaLaunchKernelEx(&cfg, fl_bwd_ss_kernel<kLayoutG128, 1>, tm_dy, tm_us, tm_code, a);
  else
    le = wide ? cudaLaunchKernelEx(&cfg, fl_bwd_ss_kernel<kLayoutNf4Dq64, 2>, tm_dy, tm_us, tm_code, a)
              : cudaLaunchKernelEx(&cfg, fl_bwd_ss_kernel<kLayoutNf4Dq64, 1>, tm_dy, tm_us, tm_code, a);
  if (le != cudaSuccess) return set_error(FL_ERR_CUDA, "bwd gemm launch: %s", cudaGetErrorString(le));
  if (ksplit > 1) return launch_split_reduce(part, ksplit, static_cast<int64_t>(M) * K, dx, stream);
  return FL_OK;
}

}  // namespace fl
