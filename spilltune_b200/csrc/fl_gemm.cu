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
// Persistent: one CTA pair per resident cluster slot walks a static list of
// tiles; stage counters run on across tiles, so TMA prefetch and decode of the
// next tile overlap the end of the current one.  The accumulator is drained
// into a 64 KiB shared-memory staging tile and leaves by an asynchronous TMA
// store (or 16-byte stores for a grouped tile that ends inside the box).
//
// Warp roles (448 threads per CTA): warp 0 TMA producer, warp 1 TMEM owner
// (both CTAs) + MMA issuer (leader CTA only), warps 2-13 dequant producers in
// three groups of four that take turns on pairs of stages (one warp per TMEM
// lane quarter decodes the whole stage for its lanes) and drain the
// accumulator after their first stage pair of the next tile.
// Synchronisation: full[s] (local TMA bytes), afull[s] (leader only: 8 local +
// 8 peer dequant-warp arrivals), empty[s] and accum (multicast tcgen05.commit
// from the leader into both CTAs), acc_empty (leader only: 12 local + 12 peer
// epilogue-warp arrivals before the next tile's first MMA).
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
// A decode group's consecutive stages are at most 2 * kGroups apart; at most
// kStages keeps its parity waits on a ring slot within one phase.
static_assert(2 * kGroups <= kStages, "decode-group rotation longer than the stage ring");

struct GemmArgs {
  const float* scales;  // fp32 [N * K/128]
  const float* lut;     // fp32 [16]
  const float* lora;    // Blora [N, r]
  __nv_bfloat16* out;   // [M, L]
  uint32_t* status;     // device status word
  int M, N, K;          // problem dims of the frozen weight W[N,K] and tokens M
  int rank;             // 0 disables the LoRA stage
  int tma_store;        // 1: full tiles leave through the output tensor map
  // Grouped (MoE) launches: tile list {expert, first row, end row, weight tile}
  // over expert-sorted token rows, its length on the device; null for one weight.
  const int4* tiles;
  const int* tile_count;
  // Dense launches with a split reduction: ksplit > 1 slices of K / ksplit,
  // FP32 sums to part[kpart][M][N] (Y is then formed by the split reduce).
  float* part;
  int ksplit;
};

struct __align__(16) GemmBarriers {
  uint64_t full[kStages];   // TMA bytes landed
  uint64_t afull[kStages];  // leader: both CTAs' dequant warps finished the TMEM A stage
  uint64_t empty[kStages];  // MMAs reading the stage completed
  uint64_t accum;           // all MMAs of the current tile completed (one phase per tile)
  uint64_t acc_empty;       // leader: both CTAs' epilogue warps drained the accumulator
  uint32_t tmem_base;
  uint32_t abort_word;
  alignas(16) float lut[16];  // codebook copy for the decoders
};

constexpr int kYBytes = kTok * kLanes * 2;  // 64 KiB bf16 output staging tile [256 tokens][128 columns]
constexpr int kEpiWarps = 4 * kGroups;
constexpr int kSmemBytes =
    1024 /*align slack*/ + kStages * (kXBytes + kQBytes) + kYBytes + static_cast<int>(sizeof(GemmBarriers));
static_assert(kSmemBytes <= 232448, "shared memory budget");

// Tile t of the launch: grouped launches read the list; dense ones walk a
// banded order in which pairs that run at the same time cover a band of
// kGroupM token tiles x several weight tiles, so an activation tile is
// requested by a handful of pairs at once instead of by every SM.
struct Tile {
  int expert, m0, m_end, w_tile, kpart;
};
__device__ __forceinline__ Tile tile_at(const GemmArgs& args, int t, int num_w, int num_m) {
  Tile r;
  if (args.tiles != nullptr) {
    const int4 v = args.tiles[t];
    r.expert = v.x;
    r.m0 = v.y;
    r.m_end = v.z;
    r.w_tile = v.w;
    r.kpart = 0;
  } else {
    // The slices of one output tile are consecutive tiles (they run together).
    r.kpart = t % args.ksplit;
    t /= args.ksplit;
    const int band = t / (kGroupM * num_w);
    const int first_m = band * kGroupM;
    const int rows_in_band = min(kGroupM, num_m - first_m);
    const int local = t - band * kGroupM * num_w;
    r.expert = 0;
    r.m0 = (first_m + local % rows_in_band) * kTok;
    r.m_end = args.M;
    r.w_tile = local / rows_in_band;
  }
  return r;
}

// Persistent: each CTA pair walks tiles pair, pair + P, ... (P pairs in the
// grid, all resident).  The stage ring counters run on across tiles, so the
// producer prefetches the next tile while the current one finishes; the
// accumulator is drained into a shared-memory staging tile (released to the
// MMA issuer as soon as it is read) and leaves by an asynchronous TMA store.
// kLayout selects the record layout the dequant warps decode (fl_codebook.cuh).
template <int kLayout>
__global__ void __launch_bounds__(kThreads, 1)
    fl_tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_act,   // X, [M, K] bf16, box {64, 128}
                      const __grid_constant__ CUtensorMap tm_low,   // Ts, [M, 64] bf16, box {64, 128}
                      const __grid_constant__ CUtensorMap tm_code,  // payload [E*N, K/2] u8, box {32, 128}, 32B swizzle
                      const __grid_constant__ CUtensorMap tm_out,   // Y [M, N] bf16, box {128, 256}
                      const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem;                                   // kStages x 16 KiB (1024-aligned)
  uint8_t* qs = smem + kStages * kXBytes;               // kStages x 4 KiB
  __nv_bfloat16* ys = reinterpret_cast<__nv_bfloat16*>(qs + kStages * kQBytes);  // 64 KiB staging
  GemmBarriers* bars = reinterpret_cast<GemmBarriers*>(qs + kStages * kQBytes + kYBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = args.M, N = args.N, K = args.K;
  const int L = N;   // output columns (TMEM lane dimension)
  const int R = K;   // reduction dimension
  const int groups_per_row = K / 128;
  const uint32_t crank = cluster_ctarank();       // 0 = leader of the CTA pair
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_w = (L + 2 * kLanes - 1) / (2 * kLanes);
  const int num_m = (M + kTok - 1) / kTok;
  const int n_tiles = args.tiles != nullptr ? *args.tile_count : num_w * num_m * args.ksplit;
  const int n_main = R / kStageK / args.ksplit;  // stages of one tile's reduction slice
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
    mbar_init(&bars->acc_empty, 2 * kEpiWarps);
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
      int g = 0;  // stage counter over all tiles of this pair
      bool ok = true;
      bool ts_ready = false;
      for (int t = pair; t < n_tiles && ok; t += num_pairs) {
        const Tile tile = tile_at(args, t, num_w, num_m);
        const int l0 = tile.w_tile * (2 * kLanes) + static_cast<int>(crank) * kLanes;
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
            const int r0 = (tile.kpart * n_main + it) * kStageK;
            mbar_arrive_expect_tx(&bars->full[s], kXBytes + kQBytes);
            tma_load_2d(xs + s * kXBytes, &tm_act, r0, mh, &bars->full[s]);
            tma_load_2d(qs + s * kQBytes, &tm_code, r0 / 2, wrow0 + l0, &bars->full[s]);  // 128 rows x 32 B
          } else {
            // Ts is the previous launch's output (lora_down, programmatic
            // dependent launch): wait for that grid before the first read.
            if (!ts_ready) {
              griddep_wait();
              ts_ready = true;
            }
            mbar_arrive_expect_tx(&bars->full[s], kXBytes);
            tma_load_2d(xs + s * kXBytes, &tm_low, 0, mh, &bars->full[s]);
          }
        }
      }
      // Finish no earlier than the previous launch (also on the abort path).
      griddep_wait();
      // Drain: never leave the CTA with bulk copies still landing in its smem.
      for (int i = g > kStages ? g - kStages : 0; i < g; ++i) {
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
      int g = 0, tl = 0;
      bool ok = true;
      for (int t = pair; t < n_tiles && ok; t += num_pairs, ++tl) {
        // The previous tile's accumulator must have been read out by both CTAs.
        if (tl > 0 &&
            !mbar_wait_cluster(&bars->acc_empty, (tl - 1) & 1, abort_word, args.status, kStatusTimeoutAccum))
          break;
        tc_fence_after();
        for (int it = 0; it < n_iter; ++it, ++g) {
          const int s = g % kStages;
          const uint32_t ph = (g / kStages) & 1;
          // Every dequant warp of both CTAs arrives only after its own CTA's
          // TMA bytes for the stage landed, so afull covers both B halves too.
          if (!mbar_wait_cluster(&bars->afull[s], ph, abort_word, args.status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(xs + s * kXBytes));
          const uint32_t a_col = tmem_base + kAccCols + s * kAStageCols;
          const int ksteps = it < n_main ? kStageK / 16 : lora_k_steps;
          for (int kk = 0; kk < ksteps; ++kk)
            mma_ts2(tmem_base, a_col + kk * 8, bdesc + 2 * kk, idesc, (it | kk) != 0 ? 1u : 0u);
          tc_commit2_mc(&bars->empty[s], 0x3);
        }
        // Completion of every MMA of the tile (also on the abort path, so TMEM
        // is never released under an in-flight MMA).
        tc_commit2_mc(&bars->accum, 0x3);
      }
      if (tl > 0) {
        uint32_t dummy_abort = 0;
        // The last commit (phase tl-1) covers every MMA this thread issued.
        mbar_wait(&bars->accum, (tl - 1) & 1, &dummy_abort, args.status, kStatusTimeoutAccum);
      }
    }
  } else {
    // ----------------------------------- dequant producers (kGroups x 4 warps)
    // Within a group: one warp per TMEM lane quarter decodes the whole stage
    // for its 32 lanes.  Groups take turns on pairs of stages (one 128-wide
    // scale group), so each warp has kGroups pair-times to hide its barrier,
    // shared-memory and TMEM-store latencies.  After the tile's last stage
    // the same warps drain the accumulator.  Every epilogue warp walks every
    // tile of the pair (also after an abort) so the named barriers match.
    const int dw = warp - 2;                   // dequant warp index
    const int grp = dw >> 2;                   // stage-pair group of this warp
    const int quarter = warp & 3;              // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;       // lane within the 128-lane tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t afull_leader = mapa_shared(smem_u32(&bars->afull[0]), 0);
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(&bars->acc_empty), 0);
    const float* lut_s = bars->lut;
    const bool elected = dw == 0 && lane == 0;  // issues and retires the output TMA stores
    bool ok = true;

    // Epilogue of tile `tile` (the pair's tl-th): drain the accumulator into
    // the staging tile, release it to the MMA issuer, store.
    auto epilogue = [&](const Tile& tile, int tl) {
      const int l0 = tile.w_tile * (2 * kLanes) + static_cast<int>(crank) * kLanes;
      // The staging tile is free once the previous tile's store has read it.
      if (elected) bulk_wait_group_read0();
      named_barrier_sync(1, 32 * kEpiWarps);
      bool drained = false;
      if (ok && mbar_wait_warp(&bars->accum, tl & 1, abort_word, args.status, kStatusTimeoutAccum)) {
        tc_fence_after();
        // The kGroups warps of each lane quarter take the 32-column token
        // chunks round robin: ys[token][row], or with a split reduction the
        // FP32 sums straight to part[kpart][token][n] (a warp's 32 rows n are
        // 128 contiguous bytes of each token row).
        const int n = l0 + row;
#pragma unroll 1
        for (int c = 32 * grp; c < kTok; c += 32 * kGroups) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem_base + lane_addr + c, v);
          tmem_wait_ld();
          if (args.ksplit > 1) {
            if (n < N) {
              float* dst = args.part + (static_cast<size_t>(tile.kpart) * M + tile.m0 + c) * N + n;
              const int live = min(32, M - tile.m0 - c);
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < live) dst[static_cast<size_t>(j) * N] = __uint_as_float(v[j]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) ys[(c + j) * kLanes + row] = __float2bfloat16_rn(__uint_as_float(v[j]));
          }
        }
        tc_fence_before();
        drained = true;
      } else {
        ok = false;
      }
      // Accumulator read out (or abandoned): release it to the MMA issuer.
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader);
      fence_proxy_async_smem();
      named_barrier_sync(1, 32 * kEpiWarps);
      if (!drained || args.ksplit > 1) return;
      const int rows_here = min(tile.m0 + kTok, M) - tile.m0;
      const bool partial = tile.m_end < tile.m0 + rows_here;
      if (args.tma_store && !partial) {
        if (elected) {
          tma_store_2d(&tm_out, ys, l0, tile.m0);
          bulk_commit_group();
        }
      } else {
        // Rows [m0, m_end) only (a grouped tile ends inside the box), or no
        // output tensor map: 16-byte vectors where the row allows.
        const int rows = min(tile.m_end, M) - tile.m0;
        const int tid = threadIdx.x - 64;
        const bool vec_ok = (L % 8) == 0 && ((reinterpret_cast<uintptr_t>(args.out) & 15u) == 0);
        for (int idx = tid; idx < rows * (kLanes / 8); idx += 32 * kEpiWarps) {
          const int r = idx / (kLanes / 8), cc = (idx % (kLanes / 8)) * 8;
          const int col = l0 + cc;
          const __nv_bfloat16* src = ys + r * kLanes + cc;
          __nv_bfloat16* dst = args.out + static_cast<size_t>(tile.m0 + r) * L + col;
          if (vec_ok && col + 8 <= L) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
          } else {
            for (int e = 0; e < 8 && col + e < L; ++e) dst[e] = src[e];
          }
        }
      }
    };

    // Order per tile: the group's first stage pair of this tile, then the
    // previous tile's epilogue, then the rest of this tile (see `first` below
    // for which pairs a group takes).  The first pairs of
    // all groups fill the stage ring, so the MMA issuer restarts on decoded
    // stages as soon as the accumulator is released.  Every epilogue warp
    // walks every tile of the pair (also after an abort): the named barriers
    // inside the epilogue always match.
    int g0 = 0;  // stage counter at the start of the tile
    int tl = 0;
    Tile prev{};
    const int pairs_per_tile = (n_iter + 1) / 2;  // the last one a single stage when n_iter is odd
    for (int t = pair; t < n_tiles; t += num_pairs, g0 += n_iter, ++tl) {
      const Tile tile = tile_at(args, t, num_w, num_m);
      const int l0 = tile.w_tile * (2 * kLanes) + static_cast<int>(crank) * kLanes;
      const int wrow0 = tile.expert * N;
      // Thread owns weight row n; each stage it decodes the 64 k of the stage
      // (32 TMEM columns).
      const int n = l0 + row;
      const bool valid = n < N;
      // Scales per row: one per 128-group (layout 0) or per 64-block = per stage
      // (layout 1).  A stage pair is one group, or two blocks.
      constexpr bool kBlock64 = kLayout == kLayoutNf4Dq64;
      const int spr = kBlock64 ? 2 * groups_per_row : groups_per_row;
      // This tile's reduction slice: 128-groups [kpart * tile_groups, + tile_groups).
      const int tile_groups = n_main / 2;
      const float* srow = args.scales + static_cast<size_t>(wrow0 + (valid ? n : 0)) * spr +
                          (kBlock64 ? 2 : 1) * tile.kpart * tile_groups;
      const bool lora_here = tile.kpart == 0;  // a split sums the LoRA stage once
      // The groups take the stage pairs of the CTA pair's whole stage sequence in
      // turn (tile tl starts a new pair, number tl * pairs_per_tile), not afresh
      // per tile: consecutive stages of one group are then never more than
      // 2 * kGroups <= kStages apart, so a group never waits on a ring slot
      // whose barrier is two phases behind (the parity wait would pass).
      const int first = (grp - (tl * pairs_per_tile) % kGroups + kGroups) % kGroups;
      const int pit0 = 2 * first;
      float next_scale = (valid && first < tile_groups) ? __ldg(srow + (kBlock64 ? 2 * first : first)) : 0.0f;
      float next_scale2 = (kBlock64 && valid && first < tile_groups) ? __ldg(srow + 2 * first + 1) : 0.0f;
      for (int pit = pit0; pit < n_iter || (pit == pit0 && tl > 0); pit += 2 * kGroups) {
        if (pit < n_iter && ok) {
          ProductTable table;
          float sc_a = 0.f, sc_b = 0.f;  // layout 1: the pair's two block scales
          if (pit < n_main) {
            const int g_next = pit / 2 + kGroups;
            if constexpr (kBlock64) {
              sc_a = next_scale;
              sc_b = next_scale2;
              next_scale = (valid && g_next < tile_groups) ? __ldg(srow + 2 * g_next) : 0.0f;
              next_scale2 = (valid && g_next < tile_groups) ? __ldg(srow + 2 * g_next + 1) : 0.0f;
            } else {
              table = make_table(lut_s, next_scale);
              next_scale = (valid && g_next < tile_groups) ? __ldg(srow + g_next) : 0.0f;
            }
          }
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
            if (!mbar_wait_warp(&bars->full[s], ph, abort_word, args.status, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            uint32_t v[32];
            if (it < n_main) {
              if constexpr (kBlock64) table = make_table(lut_s, it == pit ? sc_a : sc_b);
              // Row chunk c sits at chunk c ^ ((row >> 2) & 1) (32-byte swizzle):
              // eight consecutive rows then read distinct banks.
              const uint8_t* qrow = qs + s * kQBytes + row * 32;
              const uint32_t sw = (row >> 2) & 1;
              const uint4 q0 = *reinterpret_cast<const uint4*>(qrow + (sw << 4));
              const uint4 q1 = *reinterpret_cast<const uint4*>(qrow + ((1u ^ sw) << 4));
              lookup8_l<kLayout>(table, q0.x, v + 0);
              lookup8_l<kLayout>(table, q0.y, v + 4);
              lookup8_l<kLayout>(table, q0.z, v + 8);
              lookup8_l<kLayout>(table, q0.w, v + 12);
              lookup8_l<kLayout>(table, q1.x, v + 16);
              lookup8_l<kLayout>(table, q1.y, v + 20);
              lookup8_l<kLayout>(table, q1.z, v + 24);
              lookup8_l<kLayout>(table, q1.w, v + 28);
            } else {
              // LoRA stage: A row = bf16(Blora[n, 0:64]) zero padded past the rank.
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int c0 = 2 * j, c1 = c0 + 1;
                const float a = (valid && lora_here && c0 < args.rank) ? __ldg(args.lora + static_cast<size_t>(wrow0 + n) * args.rank + c0) : 0.f;
                const float b = (valid && lora_here && c1 < args.rank) ? __ldg(args.lora + static_cast<size_t>(wrow0 + n) * args.rank + c1) : 0.f;
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
          ok = __all_sync(0xffffffffu, ok) != 0;
        }
        if (pit == pit0 && tl > 0) epilogue(prev, tl - 1);
      }
      prev = tile;
    }
    if (tl > 0) epilogue(prev, tl - 1);
    if (elected) bulk_wait_group0();
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

#include <map>
#include <mutex>
#include <utility>

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

// Number of 2-CTA clusters of `kernel` (1 CTA per SM, `smem` dynamic bytes)
// that fit on the current device at once; sets the kernel's shared-memory
// limit on first use per device.
int resident_pairs(const void* kernel, int threads, int smem, int* pairs) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> cache;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({kernel, dev});
  if (it != cache.end()) {
    *pairs = it->second;
    return FL_OK;
  }
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
  if (e != cudaSuccess || n < 1) {
    cudaGetLastError();
    return set_error(FL_ERR_CUDA, "cluster occupancy query failed: %s", cudaGetErrorString(e));
  }
  cache[{kernel, dev}] = n;
  *pairs = n;
  return FL_OK;
}

// x: [M, K] bf16 activations; ts: [M, 64] bf16 scaled low-rank activations
// (unused when rank == 0); codes/scales/lut: the frozen record W[N, K];
// blora: [N, rank] fp32; y: [M, N] bf16.
int launch_fwd_gemm(const void* x, const void* ts, const uint8_t* codes, const float* scales, const float* lut,
                    const float* blora, int rank, void* y, int M, int N, int K, uint32_t* status,
                    cudaStream_t stream, const int4* tiles, const int* tile_count, int experts, int max_tiles,
                    int layout, bool pdl, float* part, int ksplit) {
  if (layout != kLayoutG128 && layout != kLayoutNf4Dq64) return set_error(FL_ERR_ARG, "fwd gemm: unknown layout");
  if (layout != kLayoutG128 && tiles) return set_error(FL_ERR_UNSUPPORTED, "grouped launches use layout 0");
  if (ksplit < 1 || (ksplit > 1 && (tiles || !part || (K / kStageK) % (2 * ksplit) != 0)))
    return set_error(FL_ERR_ARG, "fwd gemm: invalid reduction split %d", ksplit);
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
                          K / 2, 32, 128, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  // Output tiles leave by TMA when the row pitch and base allow it.
  const bool tma_store = (N % 8) == 0 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
  CUtensorMap tm_out = tm_act;
  if (tma_store) {
    rc = make_tensor_map_2d(&tm_out, y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, N, M, static_cast<uint64_t>(N) * 2, kLanes,
                            kTok, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
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
  a.tma_store = tma_store ? 1 : 0;
  a.tiles = tiles;
  a.tile_count = tile_count;
  a.part = part;
  a.ksplit = ksplit;
  // Persistent CTA pairs (each tile: 256 W rows x 256 tokens x one reduction
  // slice), no more than can be resident at once.
  const int tiles_max =
      tiles ? max_tiles : ((N + 2 * kLanes - 1) / (2 * kLanes)) * ((M + kTok - 1) / kTok) * ksplit;
  int pairs = 0;
  const void* kfn = layout == kLayoutG128 ? reinterpret_cast<const void*>(&fl_tc_gemm_kernel<kLayoutG128>)
                                          : reinterpret_cast<const void*>(&fl_tc_gemm_kernel<kLayoutNf4Dq64>);
  if ((rc = resident_pairs(kfn, kThreads, kSmemBytes, &pairs))) return rc;
  if (pairs > tiles_max) pairs = tiles_max;
  if (pairs < 1) return FL_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
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
  cudaError_t le = layout == kLayoutG128
                       ? cudaLaunchKernelEx(&cfg, fl_tc_gemm_kernel<kLayoutG128>, tm_act, tm_low, tm_code, tm_out, a)
                       : cudaLaunchKernelEx(&cfg, fl_tc_gemm_kernel<kLayoutNf4Dq64>, tm_act, tm_low, tm_code, tm_out, a);
  if (le != cudaSuccess) return set_error(FL_ERR_CUDA, "fwd gemm launch: %s", cudaGetErrorString(le));
  if (ksplit > 1) return launch_split_reduce(part, ksplit, static_cast<int64_t>(M) * N, y, stream);
  return FL_OK;
}

}  // namespace fl
