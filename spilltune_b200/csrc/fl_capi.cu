// extern "C" entry points of libspilltune_b200 (declared in include/spilltune_b200.h).
// Argument checking happens here, before any launch; kernels live in the other
// translation units.
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>

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

}  // namespace fl

using namespace fl;

extern "C" {

int fl_version(void) { return 101; }

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

int fl_fwd(const uint16_t* X, int64_t M, int64_t K, const uint8_t* payload, const float* scales, const float* lut16,
           int64_t N, const float* A, const float* B, int rank, float scale, uint16_t* Y, void* workspace,
           size_t workspace_bytes, void* stream) {
  int rc = check_common("fl_fwd", M, N, K, rank, payload, scales, lut16);
  if (rc) return rc;
  if (!X || !Y) return set_error(FL_ERR_ARG, "fl_fwd: null X/Y");
  if (!aligned16(X)) return set_error(FL_ERR_ARG, "fl_fwd: X must be 16-byte aligned");
  if (rank > 0) {
    if (!A || !B) return set_error(FL_ERR_ARG, "fl_fwd: null LoRA factor");
    if (!workspace || workspace_bytes < fl_fwd_workspace_bytes(M, K, rank) || !aligned16(workspace))
      return set_error(FL_ERR_ARG, "fl_fwd: workspace missing, short or misaligned");
  }
  uint32_t* status = nullptr;
  if ((rc = current_status(&status))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rank > 0) {
    void* qc = static_cast<uint8_t*>(workspace) + static_cast<size_t>(M) * 128;
    rc = launch_lora_down(X, (int)M, (int)K, A, K, 1, rank, scale, workspace, qc, st);
    if (rc) return rc;
  }
  // Decode-like steps (M <= 16) are bound by the weight bytes: dedicated kernel
  // (it streams 512-wide column chunks; other K take the tile GEMM).
  if (M <= 16 && K % 512 == 0) return launch_smallm_fwd(X, workspace, payload, scales, lut16, B, rank, Y, (int)M, (int)N, (int)K, st);
  return launch_fwd_gemm(X, workspace, payload, scales, lut16, B, rank, Y, (int)M, (int)N, (int)K, status, st);
}

int fl_bwd(const uint16_t* dY, const uint16_t* X, int64_t M, int64_t N, int64_t K, const uint8_t* payload,
           const float* scales, const float* lut16, const float* A, const float* B, int rank, float scale,
           uint16_t* dX, float* dA, float* dB, int accumulate, void* workspace, size_t workspace_bytes,
           void* stream) {
  int rc = check_common("fl_bwd", M, N, K, rank, payload, scales, lut16);
  if (rc) return rc;
  if (N % 64 != 0) return set_error(FL_ERR_ARG, "fl_bwd: out_features N=%lld must be a multiple of 64", (long long)N);
  if (!dY || !dX) return set_error(FL_ERR_ARG, "fl_bwd: null dY/dX");
  if (!aligned16(dY)) return set_error(FL_ERR_ARG, "fl_bwd: dY must be 16-byte aligned");
  if (rank > 0) {
    if (!X || !A || !B || !dA || !dB) return set_error(FL_ERR_ARG, "fl_bwd: null X or LoRA factor/gradient");
    if (!aligned16(X)) return set_error(FL_ERR_ARG, "fl_bwd: X must be 16-byte aligned");
    if (!workspace || workspace_bytes < fl_bwd_workspace_bytes(M, N, K, rank) || !aligned16(workspace))
      return set_error(FL_ERR_ARG, "fl_bwd: workspace missing, short or misaligned");
  }
  uint32_t* status = nullptr;
  if ((rc = current_status(&status))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* us = static_cast<uint8_t*>(workspace);
  uint8_t* ts = us ? us + static_cast<size_t>(M) * 128 : nullptr;
  if (rank > 0) {
    uint8_t* qc_b = ts + static_cast<size_t>(M) * 128;
    uint8_t* qc_a = qc_b + lora_factor_bytes(N, rank);
    // Us = bf16(s * dY . B): Q(j, n) = B[n * rank + j]
    if ((rc = launch_lora_down(dY, (int)M, (int)N, B, 1, rank, rank, scale, us, qc_b, st))) return rc;
    // Ts = bf16(s * X . A^T): Q(j, k) = A[j * K + k]
    if ((rc = launch_lora_down(X, (int)M, (int)K, A, K, 1, rank, scale, ts, qc_a, st))) return rc;
  }
  if ((rc = launch_bwd_gemm(dY, us, payload, scales, lut16, A, rank, dX, (int)M, (int)N, (int)K, status, st)))
    return rc;
  if (rank > 0) {
    // dA[j, k] = sum_m Us[m, j] X[m, k]
    if ((rc = launch_lora_grad(X, (int)M, (int)K, us, rank, dA, 1, K, accumulate, st))) return rc;
    // dB[n, j] = sum_m dY[m, n] Ts[m, j]
    if ((rc = launch_lora_grad(dY, (int)M, (int)N, ts, rank, dB, rank, 1, accumulate, st))) return rc;
  }
  return FL_OK;
}

}  // extern "C"
