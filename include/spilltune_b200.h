/*
 * spilltune_b200 — C ABI of the B200-native frozen-linear hot path.
 *
 * Plain pointers and sizes only.  Every pointer argument is a CUDA device
 * pointer on the calling thread's current device unless stated otherwise;
 * `stream` is a cudaStream_t (NULL = legacy default stream).  Calls enqueue
 * work on `stream` and return without synchronising.  Every entry point returns
 * FL_OK (0) or an FL_ERR_* code; fl_last_error() gives the message (per thread).
 *
 * Frozen weights use the reference's unchanged group-128 record layout
 * (ram_vram_finetune/quantization/codecs.py:34-43, :55-64, :93-105):
 *   payload : uint8[ceil(numel/128) * 64], two 4-bit codes per byte, the even
 *             element in the low nibble;
 *   scales  : float32[ceil(numel/128)], one per 128 consecutive flat elements;
 *   lut16   : float32[16] codebook; element value = bf16(lut16[code] * scale).
 * For the reference's int4-sym-g128 format lut16[c] = c - 8; the NF4 group-128
 * variant passes the NF4 codebook.  A projection weight W has shape [N, K]
 * (out_features x in_features, row-major), numel = N*K.
 *
 * Activations and outputs are row-major bf16 (passed as uint16_t bit
 * patterns); LoRA factors are fp32 A[rank, K] and B[N, rank] exactly as
 * LoRAProjection stores them (ram_vram_finetune/finetune/lora.py:97-110).
 */
#ifndef SPILLTUNE_B200_H
#define SPILLTUNE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FL_OK 0
#define FL_ERR_ARG 1          /* invalid shape, alignment or null pointer */
#define FL_ERR_UNSUPPORTED 2  /* valid request this build does not implement */
#define FL_ERR_CUDA 3         /* CUDA runtime/driver error */
#define FL_ERR_DEVICE 4       /* a kernel reported a bounded-wait timeout */

#define FL_MAX_RANK 64

/* Library version (major*10000 + minor*100 + patch). */
int fl_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* fl_last_error(void);

/* Reads the device status word of the current device: 0 when every kernel so
 * far completed its pipeline, otherwise FL_STATUS_* bits of kernels whose
 * bounded waits expired.  Synchronises the device.  reset != 0 clears it. */
int fl_status(int reset, uint32_t* status_out);

/* Status bits (fl_status). */
#define FL_STATUS_TIMEOUT_FULL (1u << 0)   /* a consumer's wait for a filled stage expired */
#define FL_STATUS_TIMEOUT_EMPTY (1u << 1)  /* a producer's wait for a free stage expired */
#define FL_STATUS_TIMEOUT_ACCUM (1u << 2)  /* a wait for the accumulator expired */
#define FL_STATUS_TIMEOUT_DRAIN (1u << 3)  /* the exit-time drain of in-flight copies expired */
#define FL_STATUS_BAD_LAUNCH (1u << 4)     /* inconsistent launch data (e.g. MoE segment offsets) */
#define FL_STATUS_BAD_INPUT (1u << 5)      /* an input value outside its domain (a CE target) */

/*
 * Self-test of the kernels' bounded device waits; no counterpart in the
 * reference.  Every wait in this library on a pipeline barrier gives up after
 * 2 s of wall time, sets a status bit and lets its kernel drain and exit, so a
 * stalled pipeline becomes an error the host reads instead of a hung GPU.  This
 * runs that wait code with `limit_ns` (<= 2 s) on a barrier phase that nothing
 * completes, synchronises `stream` and reads the status word: it returns
 * FL_ERR_DEVICE with FL_STATUS_TIMEOUT_FULL set when the wait expired and the
 * kernel returned (the expected outcome), FL_OK if the wait did not give up.
 * The status word is not cleared (fl_status(1, ...) does that).
 */
int fl_wait_selftest(uint64_t limit_ns, void* stream);

/*
 * Dequantize one group-128 record into a BF16 buffer, bit-exact with the
 * reference's decode_into (ram_vram_finetune/quantization/codecs.py:158-170,
 * called per matrix by SlotSession.load, ram_vram_finetune/memory.py:224-229).
 * numel may be any positive count (ragged tail groups allowed).
 */
int fl_dequant(const uint8_t* payload, const float* scales, const float* lut16, int64_t numel,
               uint16_t* out_bf16, void* stream);

/* Scratch bytes fl_fwd needs: the scaled low-rank activations
 * Ts = bf16(s * X.A^T) (M x 64 bf16) and A converted to a bf16 hi/lo pair
 * (4 * rank' * K bytes, rank' = rank rounded up to 16, 32 or 64) with one
 * 32-bit mask of its nonzero 8-column groups per 64 columns (4 * K / 64 bytes,
 * padded to 16); 0 when rank == 0. */
size_t fl_fwd_workspace_bytes(int64_t M, int64_t K, int rank);

/* fl_fwd_workspace_bytes plus room for FP32 partial sums when the call has too
 * few 256 x 256 output tiles to occupy the GPU (few tokens or few output
 * columns, e.g. 256 tokens of a 4096-wide projection): the tile GEMM then also
 * splits its reduction over K into 2-16 slices and a second kernel adds them in
 * slice order.  Given a workspace this large, fl_fwd and fl_fwd_nf4dq split;
 * given one of fl_fwd_workspace_bytes, they do not (results then differ only
 * in the order of the FP32 sums: each slice is summed on its own).  No
 * counterpart in the reference (one cuBLAS F.linear per projection). */
size_t fl_fwd_workspace_bytes_split(int64_t M, int64_t N, int64_t K, int rank);

/*
 * Frozen projection forward with the LoRA branch
 *   Y[M,N] = X[M,K] . W^T + scale * (X . A^T) . B^T
 * Replaces LoRAProjection.forward (ram_vram_finetune/finetune/lora.py:205-220)
 * for a weight the slot holds in packed form (the reference decodes it with
 * decode_into first, memory.py:224-229), and the NF4 path's linear_cuda
 * (ram_vram_finetune/quantization/nf4_backend_cuda.py:888-917).
 * rank = 0 computes the plain frozen F.linear (dense.py:122-124 without LoRA).
 * M <= 16 with K % 512 == 0 runs a decode-step kernel bound by the weight bytes; it factors each
 * scale group out of its dot product, so its operand is bf16(lut16[c]) (exact
 * for int4-sym, the bf16-rounded codebook for NF4) and the scale multiplies
 * the FP32 partial sum; the LoRA term is added in FP32 from the bf16
 * Ts = bf16(scale * X . A^T).
 * Requires K % 128 == 0, rank <= 64, 16-byte aligned pointers, bias-free
 * projections.  workspace: >= fl_fwd_workspace_bytes(M, K, rank) bytes,
 * 16-byte aligned (may be NULL when rank == 0); fl_fwd_workspace_bytes_split
 * bytes let a call with few output tiles split its reduction.
 */
int fl_fwd(const uint16_t* X, int64_t M, int64_t K, const uint8_t* payload, const float* scales,
           const float* lut16, int64_t N, const float* A, const float* B, int rank, float scale, uint16_t* Y,
           void* workspace, size_t workspace_bytes, void* stream);

/* Scratch bytes fl_bwd needs: Us = bf16(s * dY.B) and Ts (M x 64 bf16 each)
 * and the converted factors with their masks (as for fl_fwd, over N and over
 * K); 0 when rank == 0.  A factor whose 8-column groups are zero over whole
 * 64-row units (the block-diagonal B of projections stacked over one input)
 * costs correspondingly less low-rank work. */
size_t fl_bwd_workspace_bytes(int64_t M, int64_t N, int64_t K, int rank);

/* The same for fl_bwd / fl_bwd_ts / the NF4-DQ64 backward: room for FP32
 * partial sums of dX when its 256 x 256 tiles are too few, the reduction over
 * N then split into slices (dX's summation order changes; dA and dB do not). */
size_t fl_bwd_workspace_bytes_split(int64_t M, int64_t N, int64_t K, int rank);

/*
 * Recomputed-backward of the same projection (the autograd VJP that
 * StreamingBlockFunction.backward takes, ram_vram_finetune/training/recompute.py:85-127):
 *   dX = dY . W + scale * (dY . B) . A                        (bf16 out)
 *   dA = scale * (dY . B)^T . X,  dB = scale * dY^T . (X . A^T)  (fp32 out)
 * accumulate != 0 adds into dA/dB (grad_A/grad_B.add_, recompute.py:124-127);
 * accumulate == 0 overwrites them.  dA/dB may be NULL when rank == 0.
 * M <= 16 with K % 512 == 0 runs a decode-step kernel (the scale folded into
 * bf16(dY * scale) instead of into the weight) unless rank > 0 and
 * N % 128 != 0; otherwise the tile GEMM.
 * Requires K % 128 == 0, N % 64 == 0, rank <= 64.
 */
int fl_bwd(const uint16_t* dY, const uint16_t* X, int64_t M, int64_t N, int64_t K, const uint8_t* payload,
           const float* scales, const float* lut16, const float* A, const float* B, int rank, float scale,
           uint16_t* dX, float* dA, float* dB, int accumulate, void* workspace, size_t workspace_bytes,
           void* stream);

/*
 * fl_bwd given the forward's low-rank activations Ts = bf16(scale * X . A^T)
 * ([M, 64] bf16, 128-byte rows, zero past the rank), the intermediate the
 * reference's autograd keeps from the recomputed forward for grad_B
 * (F.linear(F.linear(x, A), B) in finetune/lora.py:219-220; its backward in
 * training/recompute.py:102-127).  fl_fwd leaves exactly these bytes in the
 * first M * 128 bytes of its workspace whenever this function reads them, so
 * the results equal fl_bwd's while X . A^T is not recomputed: dX bit for bit,
 * dA and dB up to the order of their FP32 sums (both are summed with atomic
 * adds, and with rank <= 16 this entry point sums dB in the same pass over dY
 * that forms Us).
 * Ts is not read when rank == 0, or when M <= 16 with K % 512 == 0 and the
 * group-128 layout (the decode-step kernels, which form Ts themselves); it may
 * then be NULL, as it may always be (then this is fl_bwd).  Ts must be 16-byte
 * aligned.  Other arguments and the workspace as fl_bwd.
 */
int fl_bwd_ts(const uint16_t* dY, const uint16_t* X, int64_t M, int64_t N, int64_t K, const uint8_t* payload,
              const float* scales, const float* lut16, const float* A, const float* B, int rank, float scale,
              const uint16_t* Ts, uint16_t* dX, float* dA, float* dB, int accumulate, void* workspace,
              size_t workspace_bytes, void* stream);

/*
 * Same result as fl_fwd, for callers that cannot allocate device memory at
 * call time (a host binding without a device allocator, a trainer whose
 * device budget is fixed up front).  No counterpart in the reference.  It
 * allocates nothing: the scratch lives in a 12 MiB array of this library's own
 * device memory (held on every GPU that loads the library), so when rank > 0 M
 * is limited to 32768 tokens and rank' * K to 2^21 (rank' = rank rounded up to
 * 16, 32 or 64; FL_ERR_ARG beyond).  The first call on a device
 * looks up that array's address; make it before any stream capture.  The
 * address is kept for the life of the process, so after cudaDeviceReset on a
 * device this process must not call the library on that device again.  All
 * calls on a device share the array: calls whose kernels overlap on the GPU
 * race and must be serialised by the caller.
 */
int fl_fwd_noalloc(const uint16_t* X, int64_t M, int64_t K, const uint8_t* payload, const float* scales,
                   const float* lut16, int64_t N, const float* A, const float* B, int rank, float scale,
                   uint16_t* Y, void* stream);

/*
 * Grouped (MoE expert) frozen projections.  Replaces the per-expert loop of
 * moe_feed_forward (ram_vram_finetune/adapters/qwen3_moe.py:103-112: gather
 * flat[tokens], F.linear(current, gate_up_proj[e]), F.linear(., down_proj[e]))
 * and its DeepSeek twin (adapters/deepseek.py:159-177) with one launch chain
 * over all experts, plus an optional per-expert LoRA branch.
 *
 * Rows are the routed (token, slot) pairs sorted by expert; seg[0..E] (device
 * int32) are the prefix offsets of each expert's segment: seg[0] == 0,
 * seg[E] == rows, non-decreasing.  Invalid segments write nothing and set
 * FL_STATUS bit 4 (read with fl_status).  The experts' weights form one
 * stacked record: payload [E, N, K/2], scales [E, N, K/128]; LoRA factors are
 * stacked FP32 A [E, rank, K], B [E, N, rank], gradients dA/dB likewise.
 *
 * fl_grouped_fwd: Y[m] = X[m] . W_e^T + s (X[m] . A_e^T) . B_e^T for m in
 * segment e, with the same rounding as fl_fwd.  fl_grouped_bwd: dX (and, when
 * rank > 0, dA_e/dB_e summed over the expert's rows) as fl_bwd.  Workspace of
 * fl_grouped_workspace_bytes(rows, E, N, K, rank) bytes, 16-byte aligned, for
 * either call; the segment offsets are read on the device (no host sync), so
 * both calls may be captured in a CUDA graph.
 * Requires K % 128 == 0, N % 64 == 0, rank <= 64.
 */
size_t fl_grouped_workspace_bytes(int64_t rows, int experts, int64_t N, int64_t K, int rank);
int fl_grouped_fwd(const uint16_t* X, const int32_t* seg, int64_t rows, int64_t K, int experts,
                   const uint8_t* payload, const float* scales, const float* lut16, int64_t N, const float* A,
                   const float* B, int rank, float scale, uint16_t* Y, void* workspace, size_t workspace_bytes,
                   void* stream);
int fl_grouped_bwd(const uint16_t* dY, const uint16_t* X, const int32_t* seg, int64_t rows, int64_t N, int64_t K,
                   int experts, const uint8_t* payload, const float* scales, const float* lut16, const float* A,
                   const float* B, int rank, float scale, uint16_t* dX, float* dA, float* dB, int accumulate,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * bitsandbytes NF4 with double quantization, block 64 ("NF4-DQ64") — the
 * record the reference's Qwen3.5 NF4 path stages (CUDARecord,
 * ram_vram_finetune/quantization/nf4_backend_cuda.py:522-644, layout checked
 * at nf4_backend.py:184-278) and multiplies with bnb.matmul_4bit in
 * linear_cuda (nf4_backend_cuda.py:888-917).  Layout: packed uint8
 * [(N*K+1)/2], element 2i in the HIGH nibble of byte i and 2i+1 in the low
 * nibble; absmax uint8 [ceil(N*K/64)]; nested_absmax fp32 [ceil(blocks/256)];
 * nested_map fp32[256]; quant_map fp32[16]; nested_offset >= 0.
 * bitsandbytes is not available to pin these numerics (the decode below is a
 * restatement of its published format).
 *
 * fl_nf4dq_scales: the double-quantization prologue, FP32 block scales
 *   scales[b] = fp32(nested_map[absmax[b]] * nested_absmax[b / 256]) + offset.
 * fl_dequant_nf4dq: w[i] = bf16_rne(fp32(quant_map[code_i] * scales[i / 64])).
 * fl_fwd_nf4dq / fl_bwd_nf4dq: fl_fwd / fl_bwd on such a record (block_scales
 * from fl_nf4dq_scales, computed once per staged record), same workspace
 * sizes, same LoRA branch; every M takes the tile GEMM.
 * Requires K % 128 == 0 (and N % 64 == 0 for the backward), packed 16-byte
 * aligned.
 */
int fl_nf4dq_scales(const uint8_t* absmax_q, const float* nested_absmax, const float* nested_map, float offset,
                    int64_t blocks, float* scales_out, void* stream);
int fl_dequant_nf4dq(const uint8_t* packed, const float* block_scales, const float* quant_map, int64_t numel,
                     uint16_t* out_bf16, void* stream);
int fl_fwd_nf4dq(const uint16_t* X, int64_t M, int64_t K, const uint8_t* packed, const float* block_scales,
                 const float* quant_map, int64_t N, const float* A, const float* B, int rank, float scale, uint16_t* Y,
                 void* workspace, size_t workspace_bytes, void* stream);
int fl_bwd_nf4dq(const uint16_t* dY, const uint16_t* X, int64_t M, int64_t N, int64_t K, const uint8_t* packed,
                 const float* block_scales, const float* quant_map, const float* A, const float* B, int rank,
                 float scale, uint16_t* dX, float* dA, float* dB, int accumulate, void* workspace,
                 size_t workspace_bytes, void* stream);
/* fl_bwd_ts for such a record: Ts as fl_fwd_nf4dq left it in the first
 * M * 128 bytes of its workspace (read whenever rank > 0: every M takes the
 * tile GEMM here). */
int fl_bwd_nf4dq_ts(const uint16_t* dY, const uint16_t* X, int64_t M, int64_t N, int64_t K, const uint8_t* packed,
                    const float* block_scales, const float* quant_map, const float* A, const float* B, int rank,
                    float scale, const uint16_t* Ts, uint16_t* dX, float* dA, float* dB, int accumulate,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Chunked LM head + shifted cross-entropy, one token chunk per call: the body
 * of the reference's _ChunkedCE.forward loop (ram_vram_finetune/quantization/
 * native_terminal.py:20-28; the same loop inline in training/engine.py:58-78).
 *   h       bf16 [T, H]   normalized hidden states of the chunk's tokens;
 *   head    bf16 [V, H]   frozen LM head;
 *   targets int64 [T]     next-token labels, -100 = no loss for that token;
 *                         any other value outside [0, V) adds no loss, gets a
 *                         zero gradient row and sets FL_STATUS bit 5 (read
 *                         with fl_status; the reference's F.cross_entropy
 *                         raises for it);
 *   loss_sum fp32 scalar (device) += sum over targeted tokens of
 *            logsumexp(logits) - logits[target], logits = bf16(h . head^T);
 *   dh      bf16 [T, H]   = d(loss / normalization) / dh, inv_norm = 1/normalization.
 * workspace: >= fl_ce_workspace_bytes(T, V) bytes, 256-byte aligned (holds the
 * chunk's bf16 logits).  Requires H % 8 == 0, V % 8 == 0.
 */
size_t fl_ce_workspace_bytes(int64_t T, int64_t V);
int fl_ce_chunk(const uint16_t* h, int64_t T, int64_t H, const uint16_t* head, int64_t V, const int64_t* targets,
                float inv_norm, float* loss_sum, uint16_t* dh, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPILLTUNE_B200_H */
