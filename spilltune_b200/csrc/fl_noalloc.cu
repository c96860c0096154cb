// fl_fwd_noalloc: the frozen-projection forward for callers that cannot
// allocate device memory when they call it.
//
// fl_fwd needs scratch for the scaled low-rank activations Ts = bf16(s*X.A^T)
// (M x 64 bf16) and the converted factor A, and asks the caller for it.  Some callers have no way to
// provide it: a host binding (Go/Java/C FFI) that owns no device allocator, a
// trainer that has committed its whole device budget up front and must not
// grow it per call, or code that wants no allocator traffic between kernels.
// This entry point takes the scratch from a fixed array in this library's own
// device memory instead, so it allocates nothing at all.
//
// Rules of use:
//  * Limits: M * 128 bytes must fit in kNoAllocScratchBytes (4 MiB), i.e.
//    M <= 32768 tokens per call, and the converted factor A (4 * rank' * K
//    bytes, rank' = rank rounded up to 16/32/64) in kNoAllocFactorBytes
//    (8 MiB); larger calls are rejected with FL_ERR_ARG.
//  * Every GPU that loads the library holds the 12 MiB array until exit.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current.  Make that first call
//    before any stream capture.  The address is kept for the life of the
//    process: after cudaDeviceReset on a device (which frees the module's
//    device memory), this process must not call the library on that device
//    again.
//  * All calls on a device share the one array and it keeps the last call's
//    contents.  Calls whose kernels overlap on the GPU (different streams
//    without ordering between them) race on it; serialise them.  Nothing in the
//    array needs to start at zero: each call writes every row it later reads.
#include <cuda_runtime.h>
#include <cstdint>
#include <mutex>

#include "fl_host.h"

namespace fl {

constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr size_t kNoAllocFactorBytes = 8u << 20;

// Host code must not use this name as a device address: on the host it is only
// a stand-in symbol.  Device addresses come from cudaGetSymbolAddress below.
// The first kNoAllocScratchBytes hold Ts, the rest the converted factor A.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes + kNoAllocFactorBytes];

static uint8_t* noalloc_scratch(int device) {
  static std::mutex mu;
  static uint8_t* addr[64] = {nullptr};
  if (device < 0 || device >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      set_error(FL_ERR_CUDA, "fl_fwd_noalloc: cudaGetSymbolAddress on device %d: %s", device, cudaGetErrorString(e));
      return nullptr;
    }
    addr[device] = static_cast<uint8_t*>(p);
  }
  return addr[device];
}

}  // namespace fl

using namespace fl;

extern "C" int fl_fwd_noalloc(const uint16_t* X, int64_t M, int64_t K, const uint8_t* payload, const float* scales,
                              const float* lut16, int64_t N, const float* A, const float* B, int rank, float scale,
                              uint16_t* Y, void* stream) {
  if (M <= 0 || N <= 0 || K <= 0) return set_error(FL_ERR_ARG, "fl_fwd_noalloc: dims must be positive");
  if (M > (1 << 30) || N > (1 << 30) || K > (1 << 30)) return set_error(FL_ERR_ARG, "fl_fwd_noalloc: dims too large");
  if (rank > 0 && static_cast<uint64_t>(M) * 128u > kNoAllocScratchBytes)
    return set_error(FL_ERR_ARG, "fl_fwd_noalloc: M=%lld tokens exceeds the %zu-byte scratch (max %zu tokens)",
                     (long long)M, kNoAllocScratchBytes, kNoAllocScratchBytes / 128);
  if (rank > 0 && rank <= FL_MAX_RANK && K > 0 && lora_factor_bytes(K, rank) > kNoAllocFactorBytes)
    return set_error(FL_ERR_ARG, "fl_fwd_noalloc: K=%lld at rank %d exceeds the %zu-byte factor scratch",
                     (long long)K, rank, kNoAllocFactorBytes);
  if (K % 128 != 0) return set_error(FL_ERR_ARG, "fl_fwd_noalloc: in_features K=%lld must be a multiple of 128", (long long)K);
  if (rank < 0 || rank > FL_MAX_RANK) return set_error(FL_ERR_UNSUPPORTED, "fl_fwd_noalloc: rank %d outside [0, %d]", rank, FL_MAX_RANK);
  if (!X || !Y || !payload || !scales || !lut16) return set_error(FL_ERR_ARG, "fl_fwd_noalloc: null pointer");
  if ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(payload)) & 15u)
    return set_error(FL_ERR_ARG, "fl_fwd_noalloc: X and payload must be 16-byte aligned");
  if (rank > 0 && (!A || !B)) return set_error(FL_ERR_ARG, "fl_fwd_noalloc: null LoRA factor");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "fl_fwd_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  uint32_t* status = status_word(dev);
  if (!status) return set_error(FL_ERR_CUDA, "fl_fwd_noalloc: status word unavailable on device %d", dev);
  uint8_t* ts = nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rank > 0) {
    ts = noalloc_scratch(dev);
    if (!ts) return FL_ERR_CUDA;
  }
  if (M <= 16 && K % 512 == 0) {
    // LoRA partial sums (M * 64 * K/128 floats) in the factor scratch.
    float* parts = rank > 0 ? reinterpret_cast<float*>(ts + kNoAllocScratchBytes) : nullptr;
    if (rank > 0) {
      const int rc = launch_lora_parts(X, (int)M, (int)K, A, K, 1, rank, parts, st);
      if (rc) return rc;
    }
    return launch_smallm_fwd(X, parts, scale, payload, scales, lut16, B, rank, Y, (int)M, (int)N, (int)K, st);
  }
  if (rank > 0) {
    const int rc = launch_lora_down(X, (int)M, (int)K, A, K, 1, rank, scale, ts, ts + kNoAllocScratchBytes, st);
    if (rc) return rc;
  }
  return launch_fwd_gemm(X, ts, payload, scales, lut16, B, rank, Y, (int)M, (int)N, (int)K, status, st, nullptr,
                         nullptr, 1, 0, 0, /*pdl=*/true);
}
