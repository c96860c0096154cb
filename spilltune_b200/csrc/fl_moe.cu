// Grouped (MoE expert) frozen projections over router-sorted token segments.
//
// The reference runs each routed expert as its own small F.linear over the
// tokens routed to it (ram_vram_finetune/adapters/qwen3_moe.py:95-113,
// adapters/deepseek.py:159-177).  Here the caller sorts the routed rows by
// expert once; seg[0..E] are the prefix offsets of the experts' segments in
// that order (on the device, so no host synchronisation).  A one-CTA plan
// kernel turns seg into a tile list — {expert, first row, end row, column
// tile} — and the dense kernels (forward GEMM, backward GEMM, lora_down,
// lora_grad) each run one listed tile per CTA (pair), reading the expert's
// rows of the stacked [E, N, K] packed record and its slice of the stacked
// LoRA factors.  Grids are sized for the largest tile count the segment
// lengths allow; CTAs past the planned count exit at once.
#include <cuda_runtime.h>
#include <cstdint>

#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {

namespace {

constexpr int kPlanThreads = 1024;

// Tiles of `rows` rows x `col_tiles` column tiles per expert segment, in
// expert order; inside an expert the row tile varies fastest.
__global__ void __launch_bounds__(kPlanThreads) moe_plan_kernel(const int* __restrict__ seg, int experts,
                                                               int total_rows, int rows, int col_tiles,
                                                               int4* __restrict__ tiles, int max_tiles,
                                                               int* __restrict__ count, uint32_t* status) {
  __shared__ int warp_sum[kPlanThreads / 32];
  __shared__ int carry;
  __shared__ int bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    carry = 0;
    bad = (seg[0] != 0 || seg[experts] != total_rows) ? 1 : 0;
  }
  __syncthreads();
  for (int base = 0; base < experts; base += kPlanThreads) {
    const int e = base + tid;
    int s0 = 0, s1 = 0, n = 0;
    if (e < experts) {
      s0 = seg[e];
      s1 = seg[e + 1];
      if (s1 < s0 || s0 < 0 || s1 > total_rows) {
        bad = 1;
      } else {
        n = (s1 - s0 + rows - 1) / rows * col_tiles;
      }
    }
    // Block-wide exclusive scan of n.
    int incl = n;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += v;
    }
    if (lane == 31) warp_sum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sum[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += v;
      }
      warp_sum[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int before = carry + (warp > 0 ? warp_sum[warp - 1] : 0) + incl - n;
    const int mt = (s1 - s0 + rows - 1) / rows;
    for (int i = 0; i < n; ++i) {
      const int slot = before + i;
      if (slot >= max_tiles) break;
      const int r = i % mt, c = i / mt;
      const int first = s0 + r * rows;
      tiles[slot] = make_int4(e, first, min(first + rows, s1), c);
    }
    __syncthreads();
    if (tid == 0) carry += warp_sum[kPlanThreads / 32 - 1];
    __syncthreads();
  }
  if (tid == 0) {
    if (bad || carry > max_tiles) {
      *count = 0;  // every grouped kernel then exits without touching its outputs
      atomicOr(status, kStatusBadLaunch);
    } else {
      *count = carry;
    }
  }
}

}  // namespace

int moe_max_tiles(int total_rows, int experts, int rows, int col_tiles) {
  // sum_e ceil(len_e / rows) <= total_rows / rows + experts
  return (total_rows / rows + experts) * col_tiles;
}

int launch_moe_plan(const int* seg, int experts, int total_rows, int rows, int col_tiles, int4* tiles,
                    int max_tiles, int* count, uint32_t* status, cudaStream_t stream) {
  moe_plan_kernel<<<1, kPlanThreads, 0, stream>>>(seg, experts, total_rows, rows, col_tiles, tiles, max_tiles,
                                                  count, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "moe plan launch: %s", cudaGetErrorString(e));
  return FL_OK;
}

}  // namespace fl

using namespace fl;

namespace {

constexpr int kFwdRows = 256;   // forward GEMM pair tile: 256 tokens x 256 output columns
constexpr int kBwdRows = 256;   // backward GEMM pair tile: 256 tokens x 256 input columns
constexpr int kBwdWideRows = 512;  // ... or 512 tokens when the experts average >= 384 rows
constexpr int kDownRows = 128;  // lora_down tile
constexpr int kGradRows = 512;  // lora_grad token slice

size_t align16(size_t v) { return (v + 15) / 16 * 16; }

struct GroupedPlan {
  int fwd_tiles, bwd_tiles, down_tiles, grad_tiles;
  size_t off_fwd, off_bwd, off_down, off_grad, off_count, off_us, off_ts, off_qa, off_qb, total;
};

GroupedPlan grouped_plan(int64_t rows, int experts, int64_t N, int64_t K, int rank) {
  GroupedPlan p{};
  const int r = static_cast<int>(rows);
  p.fwd_tiles = moe_max_tiles(r, experts, kFwdRows, static_cast<int>((N + 255) / 256));
  p.bwd_tiles = moe_max_tiles(r, experts, kBwdRows, static_cast<int>((K + 255) / 256));
  p.down_tiles = rank > 0 ? moe_max_tiles(r, experts, kDownRows, 1) : 0;
  p.grad_tiles = rank > 0 ? moe_max_tiles(r, experts, kGradRows, 1) : 0;
  size_t off = 0;
  p.off_fwd = off;
  off += align16(16u * p.fwd_tiles);
  p.off_bwd = off;
  off += align16(16u * p.bwd_tiles);
  p.off_down = off;
  off += align16(16u * p.down_tiles);
  p.off_grad = off;
  off += align16(16u * p.grad_tiles);
  p.off_count = off;
  off += 16;
  p.off_us = off;
  off += rank > 0 ? static_cast<size_t>(rows) * 128 : 0;
  p.off_ts = off;
  off += rank > 0 ? static_cast<size_t>(rows) * 128 : 0;
  // Converted factors of every expert: A (reduction K) and B^T (reduction N).
  p.off_qa = off;
  off += rank > 0 ? static_cast<size_t>(experts) * lora_factor_bytes(K, rank) : 0;
  p.off_qb = off;
  off += rank > 0 ? static_cast<size_t>(experts) * lora_factor_bytes(N, rank) : 0;
  p.total = off;
  return p;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_grouped(const char* who, int64_t rows, int64_t N, int64_t K, int experts, int rank, const int32_t* seg,
                  const void* payload, const float* scales, const float* lut16) {
  if (rows <= 0 || N <= 0 || K <= 0 || experts <= 0) return set_error(FL_ERR_ARG, "%s: dims must be positive", who);
  if (rows > (1 << 28) || N > (1 << 24) || K > (1 << 24) || experts > 65536)
    return set_error(FL_ERR_ARG, "%s: dims too large", who);
  if (N * experts > (int64_t(1) << 31) - 1) return set_error(FL_ERR_ARG, "%s: experts x N too large", who);
  if (K % 128 != 0) return set_error(FL_ERR_ARG, "%s: in_features K=%lld must be a multiple of 128", who, (long long)K);
  if (N % 64 != 0)
    return set_error(FL_ERR_ARG, "%s: out_features N=%lld must be a multiple of 64", who, (long long)N);
  if (rank < 0 || rank > FL_MAX_RANK)
    return set_error(FL_ERR_UNSUPPORTED, "%s: rank %d outside [0, %d]", who, rank, FL_MAX_RANK);
  if (!seg) return set_error(FL_ERR_ARG, "%s: null segment offsets", who);
  if (!payload || !scales || !lut16) return set_error(FL_ERR_ARG, "%s: null weight record pointer", who);
  if (!aligned16(payload)) return set_error(FL_ERR_ARG, "%s: payload must be 16-byte aligned", who);
  return FL_OK;
}

int grouped_status(uint32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  *out = status_word(dev);
  if (!*out) return set_error(FL_ERR_CUDA, "status word unavailable on device %d", dev);
  return FL_OK;
}

}  // namespace

extern "C" {

size_t fl_grouped_workspace_bytes(int64_t rows, int experts, int64_t N, int64_t K, int rank) {
  if (rows <= 0 || experts <= 0 || N <= 0 || K <= 0 || rank < 0) return 0;
  return grouped_plan(rows, experts, N, K, rank).total;
}

int fl_grouped_fwd(const uint16_t* X, const int32_t* seg, int64_t rows, int64_t K, int experts,
                   const uint8_t* payload, const float* scales, const float* lut16, int64_t N, const float* A,
                   const float* B, int rank, float scale, uint16_t* Y, void* workspace, size_t workspace_bytes,
                   void* stream) {
  int rc = check_grouped("fl_grouped_fwd", rows, N, K, experts, rank, seg, payload, scales, lut16);
  if (rc) return rc;
  if (!X || !Y) return set_error(FL_ERR_ARG, "fl_grouped_fwd: null X/Y");
  if (!aligned16(X)) return set_error(FL_ERR_ARG, "fl_grouped_fwd: X must be 16-byte aligned");
  if (rank > 0 && (!A || !B)) return set_error(FL_ERR_ARG, "fl_grouped_fwd: null LoRA factor");
  const GroupedPlan p = grouped_plan(rows, experts, N, K, rank);
  if (!workspace || workspace_bytes < p.total || !aligned16(workspace))
    return set_error(FL_ERR_ARG, "fl_grouped_fwd: workspace missing, short or misaligned");
  uint32_t* status = nullptr;
  if ((rc = grouped_status(&status))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int4* t_fwd = reinterpret_cast<int4*>(ws + p.off_fwd);
  int4* t_down = reinterpret_cast<int4*>(ws + p.off_down);
  int* counts = reinterpret_cast<int*>(ws + p.off_count);
  void* ts = ws + p.off_ts;
  const int r = static_cast<int>(rows), n = static_cast<int>(N), k = static_cast<int>(K);
  if ((rc = launch_moe_plan(seg, experts, r, kFwdRows, (n + 255) / 256, t_fwd, p.fwd_tiles, counts + 0, status, st)))
    return rc;
  if (rank > 0) {
    if ((rc = launch_moe_plan(seg, experts, r, kDownRows, 1, t_down, p.down_tiles, counts + 1, status, st))) return rc;
    // Ts = bf16(s * X . A_e^T), A_e = A + e * rank * K
    if ((rc = launch_lora_down(X, r, k, A, K, 1, rank, scale, ts, ws + p.off_qa, st, t_down, counts + 1,
                               p.down_tiles, static_cast<int64_t>(rank) * K, experts)))
      return rc;
  }
  return launch_fwd_gemm(X, rank > 0 ? ts : nullptr, payload, scales, lut16, B, rank, Y, r, n, k, status, st, t_fwd,
                         counts + 0, experts, p.fwd_tiles);
}

int fl_grouped_bwd(const uint16_t* dY, const uint16_t* X, const int32_t* seg, int64_t rows, int64_t N, int64_t K,
                   int experts, const uint8_t* payload, const float* scales, const float* lut16, const float* A,
                   const float* B, int rank, float scale, uint16_t* dX, float* dA, float* dB, int accumulate,
                   void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_grouped("fl_grouped_bwd", rows, N, K, experts, rank, seg, payload, scales, lut16);
  if (rc) return rc;
  if (!dY || !dX) return set_error(FL_ERR_ARG, "fl_grouped_bwd: null dY/dX");
  if (!aligned16(dY)) return set_error(FL_ERR_ARG, "fl_grouped_bwd: dY must be 16-byte aligned");
  if (rank > 0) {
    if (!X || !A || !B || !dA || !dB) return set_error(FL_ERR_ARG, "fl_grouped_bwd: null X or LoRA factor/gradient");
    if (!aligned16(X)) return set_error(FL_ERR_ARG, "fl_grouped_bwd: X must be 16-byte aligned");
  }
  const GroupedPlan p = grouped_plan(rows, experts, N, K, rank);
  if (!workspace || workspace_bytes < p.total || !aligned16(workspace))
    return set_error(FL_ERR_ARG, "fl_grouped_bwd: workspace missing, short or misaligned");
  uint32_t* status = nullptr;
  if ((rc = grouped_status(&status))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int4* t_bwd = reinterpret_cast<int4*>(ws + p.off_bwd);
  int4* t_down = reinterpret_cast<int4*>(ws + p.off_down);
  int4* t_grad = reinterpret_cast<int4*>(ws + p.off_grad);
  int* counts = reinterpret_cast<int*>(ws + p.off_count);
  uint8_t* us = rank > 0 ? ws + p.off_us : nullptr;
  uint8_t* ts = rank > 0 ? ws + p.off_ts : nullptr;
  const int r = static_cast<int>(rows), n = static_cast<int>(N), k = static_cast<int>(K);
  // Experts averaging >= 384 rows over a long reduction: 512-token tiles, each decoded
  // W stage feeding both accumulators (the plan's tile count can only fall, so
  // p.bwd_tiles still bounds it).
  const bool wide = static_cast<int64_t>(rows) >= 384LL * experts && N >= kBwdWideMinN;
  if ((rc = launch_moe_plan(seg, experts, r, wide ? kBwdWideRows : kBwdRows, (k + 255) / 256, t_bwd, p.bwd_tiles,
                            counts + 0, status, st)))
    return rc;
  bool db_done = false;
  if (rank > 0) {
    if ((rc = launch_moe_plan(seg, experts, r, kDownRows, 1, t_down, p.down_tiles, counts + 1, status, st))) return rc;
    if ((rc = launch_moe_plan(seg, experts, r, kGradRows, 1, t_grad, p.grad_tiles, counts + 2, status, st))) return rc;
    // Ts = bf16(s * X . A_e^T): Q(j, k) = A_e[j * K + k]
    if ((rc = launch_lora_down(X, r, k, A, K, 1, rank, scale, ts, ws + p.off_qa, st, t_down, counts + 1,
                               p.down_tiles, static_cast<int64_t>(rank) * K, experts)))
      return rc;
    // Us = bf16(s * dY . B_e): Q(j, n) = B_e[n * rank + j], B_e = B + e * N * rank; with
    // rank <= 16 the same pass over dY adds dB_e[n, j] += sum_{m in e} dY[m, n] Ts[m, j].
    if (!accumulate) {
      const cudaError_t e = cudaMemsetAsync(dB, 0, static_cast<size_t>(experts) * N * rank * sizeof(float), st);
      if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "fl_grouped_bwd: dB clear: %s", cudaGetErrorString(e));
    }
    if ((rc = launch_lora_down(dY, r, n, B, 1, rank, rank, scale, us, ws + p.off_qb, st, t_down, counts + 1,
                               p.down_tiles, static_cast<int64_t>(N) * rank, experts, false, ts, dB, &db_done)))
      return rc;
  }
  if ((rc = launch_bwd_gemm(dY, us, payload, scales, lut16, A, rank, dX, r, n, k, status, st, t_bwd, counts + 0,
                            experts, p.bwd_tiles, /*layout=*/0, /*pdl=*/false, nullptr, 1, wide)))
    return rc;
  if (rank > 0) {
    // dA_e[j, k] = sum_{m in e} Us[m, j] X[m, k]
    if ((rc = launch_lora_grad(X, r, k, us, rank, dA, 1, K, accumulate, st, t_grad, counts + 2, p.grad_tiles,
                               static_cast<int64_t>(rank) * K, static_cast<int64_t>(experts) * rank * K)))
      return rc;
    // dB_e[n, j] = sum_{m in e} dY[m, n] Ts[m, j], unless the Us pass summed it (it was
    // cleared above, so this adds into it)
    if (!db_done && (rc = launch_lora_grad(dY, r, n, ts, rank, dB, rank, 1, 1, st, t_grad, counts + 2,
                                           p.grad_tiles, static_cast<int64_t>(N) * rank,
                                           static_cast<int64_t>(experts) * N * rank)))
      return rc;
  }
  return FL_OK;
}

}  // extern "C"
