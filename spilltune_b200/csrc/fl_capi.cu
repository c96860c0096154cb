// extern "C" entry points of libspilltune_b200 (declared in include/spilltune_b200.h).
// Argument checking happens here, before any launch; kernels live in the other
// translation units.
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "fl_codebook.cuh"
#include "fl_host.h"

namespace fl {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

// One status word per device, in the module's static device memory.
static __device__ uint32_t g_status_word;

uint32_t* status_word(int device) {
  static std::mutex mu;
  static uint32_t* addr[64] = {nullptr};
  if (device < 0 || device >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[device]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    addr[device] = static_cast<uint32_t*>(p);
  }
  return addr[device];
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int current_status(uint32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  *out = status_word(dev);
  if (!*out) return set_error(FL_ERR_CUDA, "status word unavailable on device %d", dev);
  return FL_OK;
}

// Self-test of the bounded waits every pipeline uses (mbar_wait_warp): one CTA
// waits, with the given limit, on an mbarrier phase that nothing completes.
// Every lane's wait gives up, sets kStatusTimeoutFull in *status and returns;
// the phase is then completed so the barrier is not left pending at exit.
__global__ void wait_selftest_kernel(uint64_t limit_ns, uint32_t* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t abort_word;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_word = 0u;
    fence_barrier_init();
  }
  __syncthreads();
  (void)mbar_wait_warp(&bar, 0, &abort_word, status, kStatusTimeoutFull, limit_ns);
  __syncthreads();
  if (threadIdx.x == 0) mbar_arrive(&bar);
}

}  // namespace fl

using namespace fl;

extern "C" {

int fl_version(void) { return 310; }  // 0.3.1: reduction splits (fl_*_workspace_bytes_split)

int fl_wait_selftest(uint64_t limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > kWaitLimitNs)
    return set_error(FL_ERR_ARG, "fl_wait_selftest: limit must be in (0, %llu] ns", (unsigned long long)kWaitLimitNs);
  uint32_t* w = nullptr;
  int rc = current_status(&w);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  wait_selftest_kernel<<<1, 64, 0, st>>>(limit_ns, w);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "fl_wait_selftest: %s", cudaGetErrorString(e));
  uint32_t v = 0;
  e = cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "fl_wait_selftest: status read: %s", cudaGetErrorString(e));
  if (v & kStatusTimeoutFull)
    return set_error(FL_ERR_DEVICE, "fl_wait_selftest: bounded wait expired after %llu ns (status 0x%x)",
                     (unsigned long long)limit_ns, v);
  return set_error(FL_OK, "");
}

const char* fl_last_error(void) { return g_err; }

int fl_status(int reset, uint32_t* status_out) {
  uint32_t* w = nullptr;
  int rc = current_status(&w);
  if (rc) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "synchronize: %s", cudaGetErrorString(e));
  uint32_t v = 0;
  e = cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
  if (reset) {
    const uint32_t z = 0;
    e = cudaMemcpy(w, &z, sizeof(z), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "status reset: %s", cudaGetErrorString(e));
  }
  if (status_out) *status_out = v;
  return FL_OK;
}

int fl_dequant(const uint8_t* payload, const float* scales, const float* lut16, int64_t numel, uint16_t* out_bf16,
               void* stream) {
  if (numel < 0) return set_error(FL_ERR_ARG, "fl_dequant: negative numel");
  if (numel == 0) return FL_OK;
  if (!payload || !scales || !lut16 || !out_bf16) return set_error(FL_ERR_ARG, "fl_dequant: null pointer");
  return launch_dequant(payload, scales, lut16, numel, out_bf16, static_cast<cudaStream_t>(stream));
}

// fl_fwd workspace: [Ts: M x 64 bf16][A converted: lora_factor_bytes(K)]
size_t fl_fwd_workspace_bytes(int64_t M, int64_t K, int rank) {
  if (rank <= 0 || M <= 0 || K <= 0) return 0;
  return static_cast<size_t>(M) * 128 + lora_factor_bytes(K, rank);
}

// fl_bwd workspace: [Us][Ts] (M x 64 bf16 each) [B^T converted: N][A converted: K]
size_t fl_bwd_workspace_bytes(int64_t M, int64_t N, int64_t K, int rank) {
  if (rank <= 0 || M <= 0 || N <= 0 || K <= 0) return 0;
  return static_cast<size_t>(M) * 256 + lora_factor_bytes(N, rank) + lora_factor_bytes(K, rank);
}

}  // extern "C"

// Reduction splits of the tile GEMMs (fl_split.cu): output tiles x splits
// fill the CTA pairs when the output alone has too few tiles.  The FP32
// partial sums sit after the call's other scratch, 256-byte aligned.
static size_t align256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

static bool small_m_path(int layout, int64_t M, int64_t K);

// The GEMM is launched while the chain's low-rank kernels still run (it waits
// for their output only at its LoRA stage), so their CTAs take SMs first: the
// split keeps the GEMM's pairs within the SMs they leave, or a second wave of
// pairs would finish last.
static int pairs_beside(int lowrank_ctas) {
  const int p = device_pairs() - (lowrank_ctas + 1) / 2;
  return p > 1 ? p : 1;
}

static int fwd_ksplit(int layout, int64_t M, int64_t N, int64_t K, int rank) {
  if (M <= 0 || N <= 0 || K <= 0 || K % 128 != 0 || M > (1 << 30) || small_m_path(layout, M, K)) return 1;
  const int ld = rank > 0 ? lora_down_ctas((int)M, (int)K, rank) : 0;
  return gemm_ksplit(((N + 255) / 256) * ((M + 255) / 256), K / 64, pairs_beside(ld), device_pairs());
}

// Counted for the low-rank pass over dY that precedes the GEMM when the caller
// passes the forward's Ts (fl_bwd_ts, the autograd path; fl_bwd runs a second
// one over X beside it).  Both entry points split alike, so their dX stay
// bit-identical.
static int bwd_ksplit(int layout, int64_t M, int64_t N, int64_t K, int rank) {
  if (M <= 0 || N <= 0 || K <= 0 || N % 64 != 0 || M > (1 << 30) || small_m_path(layout, M, K)) return 1;
  const int ld = rank > 0 ? lora_down_ctas((int)M, (int)N, rank) : 0;
  return gemm_ksplit(((K + 255) / 256) * ((M + 255) / 256), N / 64, pairs_beside(ld), device_pairs());
}

extern "C" {

size_t fl_fwd_workspace_bytes_split(int64_t M, int64_t N, int64_t K, int rank) {
  const size_t base = fl_fwd_workspace_bytes(M, K, rank);
  const int ks = fwd_ksplit(kLayoutG128, M, N, K, rank);
  return ks > 1 ? align256(base) + static_cast<size_t>(ks) * M * N * sizeof(float) : base;
}

size_t fl_bwd_workspace_bytes_split(int64_t M, int64_t N, int64_t K, int rank) {
  const size_t base = fl_bwd_workspace_bytes(M, N, K, rank);
  const int ks = bwd_ksplit(kLayoutG128, M, N, K, rank);
  return ks > 1 ? align256(base) + static_cast<size_t>(ks) * M * K * sizeof(float) : base;
}

static int check_common(const char* who, int64_t M, int64_t N, int64_t K, int rank, const void* payload,
                        const float* scales, const float* lut16) {
  if (M <= 0 || N <= 0 || K <= 0) return set_error(FL_ERR_ARG, "%s: dims must be positive", who);
  if (M > (1 << 30) || N > (1 << 30) || K > (1 << 30)) return set_error(FL_ERR_ARG, "%s: dims too large", who);
  if (K % 128 != 0) return set_error(FL_ERR_ARG, "%s: in_features K=%lld must be a multiple of 128", who, (long long)K);
  if (rank < 0 || rank > FL_MAX_RANK) return set_error(FL_ERR_UNSUPPORTED, "%s: rank %d outside [0, %d]", who, rank, FL_MAX_RANK);
  if (!payload || !scales || !lut16) return set_error(FL_ERR_ARG, "%s: null weight record pointer", who);
  if (!aligned16(payload)) return set_error(FL_ERR_ARG, "%s: payload must be 16-byte aligned", who);
  return FL_OK;
}

}  // extern "C"

// Forward / backward bodies shared by the two record layouts.
// The decode-step (small-M) kernels take the call: fl_fwd then leaves LoRA
// partial sums, not Ts, in its workspace, and fl_bwd_ts does not read Ts.
static bool small_m_path(int layout, int64_t M, int64_t K) {
  return layout == kLayoutG128 && M <= 16 && K % 512 == 0;
}

static int fwd_impl(const char* who, int layout, const uint16_t* X, int64_t M, int64_t K, const uint8_t* payload,
                    const float* scales, const float* lut16, int64_t N, const float* A, const float* B, int rank,
                    float scale, uint16_t* Y, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_common(who, M, N, K, rank, payload, scales, lut16);
  if (rc) return rc;
  if (!X || !Y) return set_error(FL_ERR_ARG, "%s: null X/Y", who);
  if (!aligned16(X)) return set_error(FL_ERR_ARG, "%s: X must be 16-byte aligned", who);
  if (rank > 0) {
    if (!A || !B) return set_error(FL_ERR_ARG, "%s: null LoRA factor", who);
    if (!workspace || workspace_bytes < fl_fwd_workspace_bytes(M, K, rank) || !aligned16(workspace))
      return set_error(FL_ERR_ARG, "%s: workspace missing, short or misaligned", who);
  }
  uint32_t* status = nullptr;
  if ((rc = current_status(&status))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* qc = rank > 0 ? static_cast<uint8_t*>(workspace) + static_cast<size_t>(M) * 128 : nullptr;
  // Decode-like steps (M <= 16) are bound by the weight bytes: dedicated kernel
  // (it streams 512-wide column chunks; other K take the tile GEMM).  Its LoRA
  // partial sums use the converted-factor scratch (M * 64 * K/128 floats fit).
  if (small_m_path(layout, M, K)) {
    float* parts = static_cast<float*>(qc);
    if (rank > 0 && (rc = launch_lora_parts(X, (int)M, (int)K, A, K, 1, rank, parts, st))) return rc;
    return launch_smallm_fwd(X, parts, scale, payload, scales, lut16, B, rank, Y, (int)M, (int)N, (int)K, st, layout);
  }
  if (rank > 0) {
    rc = launch_lora_down(X, (int)M, (int)K, A, K, 1, rank, scale, workspace, qc, st);
    if (rc) return rc;
  }
  // Chain prepass -> lora_down -> GEMM: each waits for the previous grid only
  // before it reads that grid's output (the GEMM: before its LoRA stage).
  // Few output tiles: also split the reduction when the caller's workspace
  // has room for the partial sums (fl_fwd_workspace_bytes_split).
  int ks = fwd_ksplit(layout, M, N, K, rank);
  float* part = nullptr;
  if (ks > 1) {
    const size_t off = align256(fl_fwd_workspace_bytes(M, K, rank));
    if (workspace && aligned16(workspace) && workspace_bytes >= off + static_cast<size_t>(ks) * M * N * sizeof(float))
      part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + off);
    else
      ks = 1;
  }
  return launch_fwd_gemm(X, workspace, payload, scales, lut16, B, rank, Y, (int)M, (int)N, (int)K, status, st,
                         nullptr, nullptr, 1, 0, layout, /*pdl=*/true, part, ks);
}

static int bwd_impl(const char* who, int layout, const uint16_t* dY, const uint16_t* X, int64_t M, int64_t N,
                    int64_t K, const uint8_t* payload, const float* scales, const float* lut16, const float* A,
                    const float* B, int rank, float scale, uint16_t* dX, float* dA, float* dB, int accumulate,
                    void* workspace, size_t workspace_bytes, void* stream, const uint16_t* ts_in = nullptr) {
  int rc = check_common(who, M, N, K, rank, payload, scales, lut16);
  if (rc) return rc;
  if (N % 64 != 0) return set_error(FL_ERR_ARG, "%s: out_features N=%lld must be a multiple of 64", who, (long long)N);
  if (!dY || !dX) return set_error(FL_ERR_ARG, "%s: null dY/dX", who);
  if (!aligned16(dY)) return set_error(FL_ERR_ARG, "%s: dY must be 16-byte aligned", who);
  if (rank > 0) {
    if (!X || !A || !B || !dA || !dB) return set_error(FL_ERR_ARG, "%s: null X or LoRA factor/gradient", who);
    if (!aligned16(X)) return set_error(FL_ERR_ARG, "%s: X must be 16-byte aligned", who);
    if (!workspace || workspace_bytes < fl_bwd_workspace_bytes(M, N, K, rank) || !aligned16(workspace))
      return set_error(FL_ERR_ARG, "%s: workspace missing, short or misaligned", who);
    if (ts_in != nullptr && !aligned16(ts_in)) return set_error(FL_ERR_ARG, "%s: Ts must be 16-byte aligned", who);
  }
  uint32_t* status = nullptr;
  if ((rc = current_status(&status))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* us = static_cast<uint8_t*>(workspace);
  uint8_t* ts = us ? us + static_cast<size_t>(M) * 128 : nullptr;
  uint8_t* qc_b = rank > 0 ? ts + static_cast<size_t>(M) * 128 : nullptr;
  uint8_t* qc_a = rank > 0 ? qc_b + lora_factor_bytes(N, rank) : nullptr;
  // Decode-like steps (M <= 16) take the small-M backward, which also finishes
  // the LoRA gradients; the tile GEMM's 256-token tiles would leave most SMs
  // idle.  Its low-rank partials use the converted-factor scratch, and its
  // reduction of dY . B runs over 128-wide pieces of N: with a LoRA branch and
  // N % 128 != 0 the tile path takes the call.  The forward of such a call ran
  // the decode-step kernel and left no Ts, so a Ts passed in is never read.
  const bool small = small_m_path(layout, M, K);
  if (small) ts_in = nullptr;
  if (small && (rank == 0 || N % 128 == 0)) {
    float* uparts = reinterpret_cast<float*>(qc_b);
    float* tparts = reinterpret_cast<float*>(qc_a);
    if (rank > 0) {
      // X . A^T over K and dY . B over N (Q(j, n) = B[n * rank + j]) in one
      // launch, which lets the backward start at once.
      if ((rc = launch_lora_parts2(X, (int)K, A, K, 1, tparts, dY, (int)N, B, 1, rank, uparts, (int)M, rank, st)))
        return rc;
    }
    return launch_smallm_bwd(dY, X, uparts, tparts, scale, payload, scales, lut16, A, rank, dX, dA, dB, accumulate,
                             (int)M, (int)N, (int)K, st);
  }
  // One chain of programmatic dependent launches after the gradient clears.
  // Given the forward's Ts: prepass(B) -> lora_down(Us; with rank <= 16 it also
  // adds dB = dY^T . Ts from the same dY tiles) -> backward GEMM -> lora_grad(dA)
  // [-> lora_grad(dB) above rank 16].  Without it: prepass(B) -> lora_down(Us) ->
  // prepass(A) -> lora_down(Ts) -> backward GEMM -> lora_grad(dA) ->
  // lora_grad(dB) (computing Ts first so that one pass could also sum dB
  // serialises the two low-rank passes, which measured slower).  A split of
  // the GEMM's reduction adds its reduce kernel right after the GEMM.  Each kernel
  // waits for the previous grid before reading what the chain produced; the
  // gradient kernels start once the GEMM has seen Us and Ts complete and fill
  // the SMs its last tiles leave idle.
  if (rank > 0 && ts_in != nullptr) ts = reinterpret_cast<uint8_t*>(const_cast<uint16_t*>(ts_in));  // read only
  if (rank > 0 && !accumulate) {
    cudaError_t e = cudaMemsetAsync(dA, 0, static_cast<size_t>(rank) * K * sizeof(float), st);
    if (e == cudaSuccess) e = cudaMemsetAsync(dB, 0, static_cast<size_t>(N) * rank * sizeof(float), st);
    if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "%s: gradient clear: %s", who, cudaGetErrorString(e));
  }
  bool db_done = false;
  if (rank > 0) {
    // Us = bf16(s * dY . B): Q(j, n) = B[n * rank + j]; given Ts, also dB[n, j] +=
    // sum_m dY[m, n] Ts[m, j] in the same pass when the rank allows it.
    const bool have_ts = ts_in != nullptr;
    if ((rc = launch_lora_down(dY, (int)M, (int)N, B, 1, rank, rank, scale, us, qc_b, st, nullptr, nullptr, 0, 0, 1,
                               /*pdl=*/false, have_ts ? ts : nullptr, have_ts ? dB : nullptr, &db_done)))
      return rc;
    // Ts = bf16(s * X . A^T): Q(j, k) = A[j * K + k], unless the caller kept
    // the forward's.
    if (!have_ts &&
        (rc = launch_lora_down(X, (int)M, (int)K, A, K, 1, rank, scale, ts, qc_a, st, nullptr, nullptr, 0, 0, 1,
                               /*pdl=*/true)))
      return rc;
  }
  // Few dX tiles: also split the reduction over N when the workspace has room
  // (fl_bwd_workspace_bytes_split); the split reduce then follows the GEMM in
  // the chain, and releases the gradient kernels at once.
  int ks = bwd_ksplit(layout, M, N, K, rank);
  float* part = nullptr;
  if (ks > 1) {
    const size_t off = align256(fl_bwd_workspace_bytes(M, N, K, rank));
    if (workspace && aligned16(workspace) && workspace_bytes >= off + static_cast<size_t>(ks) * M * K * sizeof(float))
      part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + off);
    else
      ks = 1;
  }
  if ((rc = launch_bwd_gemm(dY, us, payload, scales, lut16, A, rank, dX, (int)M, (int)N, (int)K, status, st,
                            nullptr, nullptr, 1, 0, layout, /*pdl=*/true, part, ks)))
    return rc;
  if (rank > 0) {
    // dA[j, k] = sum_m Us[m, j] X[m, k]
    if ((rc = launch_lora_grad(X, (int)M, (int)K, us, rank, dA, 1, K, 1, st, nullptr, nullptr, 0, 0, 0,
                               /*pdl=*/true)))
      return rc;
    // dB[n, j] = sum_m dY[m, n] Ts[m, j]
    if (!db_done && (rc = launch_lora_grad(dY, (int)M, (int)N, ts, rank, dB, rank, 1, 1, st, nullptr, nullptr, 0, 0,
                                           0, /*pdl=*/true)))
      return rc;
  }
  return FL_OK;
}

extern "C" {

int fl_fwd(const uint16_t* X, int64_t M, int64_t K, const uint8_t* payload, const float* scales, const float* lut16,
           int64_t N, const float* A, const float* B, int rank, float scale, uint16_t* Y, void* workspace,
           size_t workspace_bytes, void* stream) {
  return fwd_impl("fl_fwd", kLayoutG128, X, M, K, payload, scales, lut16, N, A, B, rank, scale, Y, workspace,
                  workspace_bytes, stream);
}

int fl_bwd(const uint16_t* dY, const uint16_t* X, int64_t M, int64_t N, int64_t K, const uint8_t* payload,
           const float* scales, const float* lut16, const float* A, const float* B, int rank, float scale,
           uint16_t* dX, float* dA, float* dB, int accumulate, void* workspace, size_t workspace_bytes,
           void* stream) {
  return bwd_impl("fl_bwd", kLayoutG128, dY, X, M, N, K, payload, scales, lut16, A, B, rank, scale, dX, dA, dB,
                  accumulate, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------- NF4-DQ64
int fl_nf4dq_scales(const uint8_t* absmax_q, const float* nested_absmax, const float* nested_map, float offset,
                    int64_t blocks, float* scales_out, void* stream) {
  if (blocks < 0) return set_error(FL_ERR_ARG, "fl_nf4dq_scales: negative block count");
  if (blocks == 0) return FL_OK;
  if (!absmax_q || !nested_absmax || !nested_map || !scales_out)
    return set_error(FL_ERR_ARG, "fl_nf4dq_scales: null pointer");
  if (!(offset >= 0.0f) || offset != offset) return set_error(FL_ERR_ARG, "fl_nf4dq_scales: offset must be >= 0");
  return launch_nf4dq_prologue(absmax_q, nested_absmax, nested_map, offset, blocks, scales_out,
                               static_cast<cudaStream_t>(stream));
}

int fl_dequant_nf4dq(const uint8_t* packed, const float* block_scales, const float* quant_map, int64_t numel,
                     uint16_t* out_bf16, void* stream) {
  if (numel < 0) return set_error(FL_ERR_ARG, "fl_dequant_nf4dq: negative numel");
  if (numel == 0) return FL_OK;
  if (!packed || !block_scales || !quant_map || !out_bf16) return set_error(FL_ERR_ARG, "fl_dequant_nf4dq: null pointer");
  return launch_dequant(packed, block_scales, quant_map, numel, out_bf16, static_cast<cudaStream_t>(stream),
                        kLayoutNf4Dq64);
}

int fl_bwd_ts(const uint16_t* dY, const uint16_t* X, int64_t M, int64_t N, int64_t K, const uint8_t* payload,
              const float* scales, const float* lut16, const float* A, const float* B, int rank, float scale,
              const uint16_t* Ts, uint16_t* dX, float* dA, float* dB, int accumulate, void* workspace,
              size_t workspace_bytes, void* stream) {
  return bwd_impl("fl_bwd_ts", kLayoutG128, dY, X, M, N, K, payload, scales, lut16, A, B, rank, scale, dX, dA, dB,
                  accumulate, workspace, workspace_bytes, stream, Ts);
}

int fl_bwd_nf4dq_ts(const uint16_t* dY, const uint16_t* X, int64_t M, int64_t N, int64_t K, const uint8_t* packed,
                    const float* block_scales, const float* quant_map, const float* A, const float* B, int rank,
                    float scale, const uint16_t* Ts, uint16_t* dX, float* dA, float* dB, int accumulate,
                    void* workspace, size_t workspace_bytes, void* stream) {
  return bwd_impl("fl_bwd_nf4dq_ts", kLayoutNf4Dq64, dY, X, M, N, K, packed, block_scales, quant_map, A, B, rank,
                  scale, dX, dA, dB, accumulate, workspace, workspace_bytes, stream, Ts);
}

int fl_fwd_nf4dq(const uint16_t* X, int64_t M, int64_t K, const uint8_t* packed, const float* block_scales,
                 const float* quant_map, int64_t N, const float* A, const float* B, int rank, float scale, uint16_t* Y,
                 void* workspace, size_t workspace_bytes, void* stream) {
  return fwd_impl("fl_fwd_nf4dq", kLayoutNf4Dq64, X, M, K, packed, block_scales, quant_map, N, A, B, rank, scale, Y,
                  workspace, workspace_bytes, stream);
}

int fl_bwd_nf4dq(const uint16_t* dY, const uint16_t* X, int64_t M, int64_t N, int64_t K, const uint8_t* packed,
                 const float* block_scales, const float* quant_map, const float* A, const float* B, int rank,
                 float scale, uint16_t* dX, float* dA, float* dB, int accumulate, void* workspace,
                 size_t workspace_bytes, void* stream) {
  return bwd_impl("fl_bwd_nf4dq", kLayoutNf4Dq64, dY, X, M, N, K, packed, block_scales, quant_map, A, B, rank, scale,
                  dX, dA, dB, accumulate, workspace, workspace_bytes, stream);
}

}  // extern "C"
