// Host-side internals shared by the .cu translation units of libspilltune_b200.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "spilltune_b200.h"

namespace fl {

// Records a formatted message for fl_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);

uint32_t* status_word(int device);  // device status word of the calling device

// Call chains.  `pdl` launches a kernel as a programmatic dependent of the
// previous launch of the stream, which must be the chain's producer of the
// operand named below; every kernel that can be so launched waits for the
// previous grid before it reads that operand and again before it exits, so a
// chain's completion stays ordered.  Inputs written before the chain's first
// (ordinary) launch are read without waiting.
//
// Y[M,N] = X . W^T + Ts . Blora^T (fl_gemm.cu).  pdl: Ts is the previous
// launch's (lora_down) output.
// Grouped (MoE) form: `tiles`/`tile_count` from launch_moe_plan, the weight a
// stacked [experts, N, K] record, blora [experts, N, rank]; grid sized for
// `max_tiles`.  tiles == nullptr: one weight, experts = 1.
// Split of the reduction (dense launches only): with ksplit > 1 tile t covers
// reduction stages [t.kpart * S, (t.kpart + 1) * S), S = K / 64 / ksplit, and
// writes its FP32 sums to part[kpart][M][N] instead of Y (the LoRA stage is
// summed by kpart 0 only); launch_split_reduce then forms Y.
int launch_fwd_gemm(const void* x, const void* ts, const uint8_t* codes, const float* scales, const float* lut,
                    const float* blora, int rank, void* y, int M, int N, int K, uint32_t* status,
                    cudaStream_t stream, const int4* tiles = nullptr, const int* tile_count = nullptr,
                    int experts = 1, int max_tiles = 0, int layout = 0, bool pdl = false, float* part = nullptr,
                    int ksplit = 1);

// Reduction split of a dense tile GEMM with `tiles` output tiles of `stages`
// 64-wide reduction stages: 1, or the largest power of two (<= 16) for which
// every split keeps an even number, at least 8, of stages and tiles * split
// pairs fit in `pairs_free` (the CTA pairs beside the chain's low-rank
// kernels) -- in `pairs_all` when each slice still has >= 64 stages.  No split
// below 32 stages (the reduce launch would cost more than the shorter tiles
// save).  Output tiles that would leave most pairs idle (few tokens, few
// output columns) then use them all.
int gemm_ksplit(int64_t tiles, int64_t stages, int pairs_free, int pairs_all);
int device_pairs();  // SMs / 2 of the current device (74 when it cannot be queried)
// out[i] = bf16(part[0][i] + part[1][i] + ... + part[split-1][i]), i < plane,
// summed in that order (fl_split.cu).  Launched as a programmatic dependent of
// the GEMM that wrote `part`: it releases its own dependents at once and waits
// for the previous grid before reading.
int launch_split_reduce(const float* part, int split, int64_t plane, void* out, cudaStream_t stream);

// 2-CTA clusters of `kernel` that can be resident at once on the current
// device (also raises the kernel's dynamic shared-memory limit to `smem`).
int resident_pairs(const void* kernel, int threads, int smem, int* pairs);

// Tile list over expert segments: seg[0..E] (device int32 prefix offsets of the
// expert-sorted rows); each entry {expert, first row, end row, column tile} for
// `rows` rows x `col_tiles` column tiles; count written to *count.
// Invalid segments (not monotone, seg[0] != 0 or seg[E] != total_rows) or a
// list longer than max_tiles: count = 0 and kStatusBadLaunch in *status.
int launch_moe_plan(const int* seg, int experts, int total_rows, int rows, int col_tiles, int4* tiles,
                    int max_tiles, int* count, uint32_t* status, cudaStream_t stream);
int moe_max_tiles(int total_rows, int experts, int rows, int col_tiles);

// dX[M,K] = dY . W + Us . Alora (fl_gemm_bwd.cu).  pdl: Us comes from the chain
// (the previous launch completes after it); dependents are released only once
// Us and Ts are complete (the gradient kernels read them without waiting).
// ksplit > 1 (dense only): tile t sums reduction rows n in [t.kpart * S * 64,
// (t.kpart + 1) * S * 64), S = N / 64 / ksplit, into part[kpart][M][K] (FP32;
// the LoRA stage in kpart 0 only), for launch_split_reduce.
// grouped_wide: a grouped launch whose tile list has 512-row tiles (launch_moe_plan with
// rows = 512) runs the 512-token pair tiles (the caller decides, so the plan and the
// kernel agree); dense launches choose them themselves.
constexpr int kBwdWideMinN = 64 * 64;  // 512-token backward tiles need a reduction over N >= this
int launch_bwd_gemm(const void* dy, const void* us, const uint8_t* codes, const float* scales, const float* lut,
                    const float* alora, int rank, void* dx, int M, int N, int K, uint32_t* status,
                    cudaStream_t stream, const int4* tiles = nullptr, const int* tile_count = nullptr,
                    int experts = 1, int max_tiles = 0, int layout = 0, bool pdl = false, float* part = nullptr,
                    int ksplit = 1, bool grouped_wide = false);

int launch_dequant(const uint8_t* payload, const float* scales, const float* lut, int64_t numel, void* out,
                   cudaStream_t stream, int layout = 0);
// FP32 block scales of an NF4-DQ64 record (the double-quantization prologue).
int launch_nf4dq_prologue(const uint8_t* absmax_q, const float* nested_absmax, const float* nested_map, float offset,
                          int64_t blocks, float* out, cudaStream_t stream);

// out[m, j] = bf16(s * sum_r P[m, r] * Q(j, r)), j < rank, zero for rank <= j < 64.
// Q(j, r) = q[j * q_sj + r * q_sr] (fp32).  qc_scratch: lora_factor_bytes(R,
// rank) per expert, 16-byte aligned (the converted factor).
// Grouped (MoE) form: 128-row tiles over expert-sorted rows, the factor of tile
// t at q + tiles[t].x * q_expert_stride, `experts` factors converted.
// Two launches: the factor prepass, then the projection as its programmatic
// dependent.  pdl: the prepass is itself a dependent of the previous launch
// (it reads only q, written before the chain).
// lo2 / grad / grad_done: with grad != nullptr and rank <= 16 the same pass over P
// also adds grad[r * rank + j] += sum_m P[m, r] * lo2[m * 64 + j] (lo2 bf16
// [M, 64], complete before this call; grad fp32, cleared by the caller when it
// starts a sum; grouped: expert e's rows into grad + e * q_expert_stride) and sets
// *grad_done; otherwise *grad_done stays false and the caller computes grad
// itself (launch_lora_grad).
int launch_lora_down(const void* P, int M, int R, const float* q, int64_t q_sj, int64_t q_sr, int rank,
                     float s, void* out64, void* qc_scratch, cudaStream_t stream, const int4* tiles = nullptr,
                     const int* tile_count = nullptr, int max_tiles = 0, int64_t q_expert_stride = 0,
                     int experts = 1, bool pdl = false, const void* lo2 = nullptr, float* grad = nullptr,
                     bool* grad_done = nullptr);
// Small-M form (M <= 16): parts[m][j][c] (j < rank) = sum of P[m, r] * Q(j, r),
// Q(j, r) = q[j * q_sj + r * q_sr], over the 128 * lora_parts_per_cluster(R)
// columns of partial c, exact FP32 (parts: M * 64 * R / (128 * per_cluster)
// floats).  Lets the next launch of the stream start at once (programmatic
// dependent launch).
int launch_lora_parts(const void* P, int M, int R, const float* q, int64_t q_sj, int64_t q_sr, int rank,
                      float* parts, cudaStream_t stream);
// Two such reductions over the same M rows in one launch (the backward's X·Aᵀ and
// dY·B): both use the common cluster size lora_parts_per_cluster(R0, R1), so
// partial counts are R0 / (128 * it) and R1 / (128 * it).
int launch_lora_parts2(const void* P0, int R0, const float* q0, int64_t q0_sj, int64_t q0_sr, float* parts0,
                       const void* P1, int R1, const float* q1, int64_t q1_sj, int64_t q1_sr, float* parts1, int M,
                       int rank, cudaStream_t stream);
// 128-wide pieces summed into one partial (R1 > 0: the common size for both).
int lora_parts_per_cluster(int R0, int R1 = 0);
int lora_nq(int rank);                           // rank padded to 16, 32 or 64
// CTAs of the tiled launch_lora_down grid for M rows (one per SM at most);
// 0 for the small-M form.  A tile GEMM launched as its programmatic dependent
// shares the GPU with these.
int lora_down_ctas(int M, int R, int rank);
size_t lora_factor_bytes(int64_t R, int rank);   // converted-factor scratch for a reduction of R

// out(p, j) (+)= sum_m P[m, p] * Q[m, j]  (P bf16 [M, Pdim], Q bf16 [M, 64]),
// out(p, j) = out[p * o_sp + j * o_sj] fp32, j < rank.
// Grouped (MoE) form: token slices {expert, first row, end row, 0} over
// expert-sorted rows; slice t accumulates into out + tiles[t].x * out_expert_stride
// (out then holds all experts: `out_total` floats are cleared when !accumulate).
// pdl: launched after the backward GEMM (or the split reduce that follows it)
// or another lora_grad of the chain (P and Q complete; a chain clears `out`
// before its first launch).
int launch_lora_grad(const void* P, int M, int Pdim, const void* Q, int rank, float* out, int64_t o_sp,
                     int64_t o_sj, int accumulate, cudaStream_t stream, const int4* tiles = nullptr,
                     const int* tile_count = nullptr, int max_tiles = 0, int64_t out_expert_stride = 0,
                     int64_t out_total = 0, bool pdl = false);

// Y[M,N] for M <= 16 tokens (fl_smallm.cu); K % 512 == 0, layout 0.  With rank > 0 the
// LoRA term uses Ts = bf16(s * sum of the K/128 pieces of lora_parts), and the
// launch may overlap the preceding one, which must be the launch_lora_parts
// that wrote them (programmatic dependent launch).
int launch_smallm_fwd(const void* X, const float* lora_parts, float s, const uint8_t* codes, const float* scales,
                      const float* lut, const float* lora, int rank, void* Y, int M, int N, int K,
                      cudaStream_t stream, int layout = 0);

// The whole projection backward for M <= 16 tokens (fl_smallm_bwd.cu): dX[M,K] =
// dY . W + Us . Alora and, with rank > 0, dA, dB (+= when accumulate), Us / Ts =
// bf16(s * the launch_lora_parts2 partials of X . A^T over K (job 0) and of dY . B
// over N (job 1)).  K % 512 == 0, N % 64 == 0 (N % 128 == 0 when rank > 0),
// layout 0.  With rank > 0 the launch may overlap the preceding one, which must be
// that launch_lora_parts2 (programmatic dependent launch).
int launch_smallm_bwd(const void* dY, const void* X, const float* uparts, const float* tparts, float s,
                      const uint8_t* codes, const float* scales, const float* lut, const float* alora, int rank,
                      void* dX, float* dA, float* dB, int accumulate, int M, int N, int K, cudaStream_t stream);

// Chunked LM head + cross-entropy (fl_head.cu).
size_t ce_workspace_bytes(int64_t T, int64_t V);
int launch_ce_chunk(const void* h, int T, int H, const void* head, int V, const int64_t* targets, float inv_norm,
                    float* loss_sum, void* dh, void* ws, cudaStream_t stream);

}  // namespace fl
