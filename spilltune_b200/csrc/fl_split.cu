// Split of the reduction for tile GEMMs whose output has too few 256 x 256
// tiles to occupy the GPU (few tokens, or few output columns: at 256 tokens a
// 4096-wide projection is 16 tiles for 74 CTA pairs).  The GEMM's tiles then
// also run over slices of the reduction and leave FP32 sums, which this file's
// kernel adds in slice order and rounds to bf16 once, like the unsplit
// accumulator.  Deterministic: no atomics, a fixed order of the sums.
#include <cuda_bf16.h>
#include <cstdint>

#include "fl_host.h"
#include "fl_ptx.cuh"

namespace fl {

// out[i] = bf16(part[0][i] + ... + part[S-1][i]), summed in that order.  vec:
// plane % 4 == 0 and out 8-byte aligned, so a thread moves float4 vectors (part
// is 16-byte aligned: it starts a 256-byte aligned workspace region).  Each
// step a thread issues the loads of V = 16 / S vectors of all S slices
// together (16 loads in flight: the grid is only one CTA per SM).
template <int S>
__global__ void __launch_bounds__(256) split_reduce_kernel(const float* __restrict__ part, int64_t plane,
                                                           __nv_bfloat16* __restrict__ out, int vec) {
  constexpr int V = 16 / S;
  // The next launch of a call chain (a gradient kernel) reads nothing this
  // kernel writes: let it start; then wait for the GEMM that wrote `part`.
  griddep_launch_dependents();
  griddep_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  int64_t done = 0;
  if (vec) {
    const int64_t n4 = plane / 4;
    const float4* p4 = reinterpret_cast<const float4*>(part);
    for (int64_t i0 = first; i0 < n4; i0 += V * stride) {
      float4 b[V][S];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const int64_t i = i0 + v * stride;
#pragma unroll
        for (int s = 0; s < S; ++s) b[v][s] = i < n4 ? p4[s * n4 + i] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const int64_t i = i0 + v * stride;
        float4 a = b[v][0];
#pragma unroll
        for (int s = 1; s < S; ++s) {
          a.x += b[v][s].x;
          a.y += b[v][s].y;
          a.z += b[v][s].z;
          a.w += b[v][s].w;
        }
        if (i < n4) {
          uint2 o;
          o.x = pack_bf16x2(a.x, a.y);
          o.y = pack_bf16x2(a.z, a.w);
          reinterpret_cast<uint2*>(out)[i] = o;
        }
      }
    }
    done = n4 * 4;
  }
  for (int64_t i = done + first; i < plane; i += stride) {
    float a = part[i];
#pragma unroll
    for (int s = 1; s < S; ++s) a += part[s * plane + i];
    out[i] = __float2bfloat16_rn(a);
  }
}

int gemm_ksplit(int64_t tiles, int64_t stages, int pairs_free, int pairs_all) {
  int split = 1;
  if (stages < 32) return split;
  while (split < 16 && stages % (4 * split) == 0 && stages / (2 * split) >= 8) {
    // Slices of >= 64 stages outlast the chain's low-rank kernels many times
    // over: pairs that start only once those finish still end close to the rest.
    const int limit = stages / (2 * split) >= 64 ? pairs_all : pairs_free;
    if (tiles * 2 * split > limit) break;
    split *= 2;
  }
  return split;
}

int device_pairs() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 2) {
    cudaGetLastError();
    return 74;
  }
  return sms / 2;
}

int launch_split_reduce(const float* part, int split, int64_t plane, void* out, cudaStream_t stream) {
  if (plane <= 0) return FL_OK;
  const int vec = (plane % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 7u) == 0) ? 1 : 0;
  const int64_t work = vec ? plane / 4 : plane;
  // One CTA per SM at most: the grid is launched early (programmatic dependent
  // launch) and waits; a larger one would hold the thread slots that the
  // chain's gradient kernels, released at the same time, need.
  int blocks = static_cast<int>((work + 256 - 1) / 256);
  const int cap = 2 * device_pairs();
  if (blocks > cap) blocks = cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto* o = static_cast<__nv_bfloat16*>(out);
  cudaError_t e;
  switch (split) {
    case 2: e = cudaLaunchKernelEx(&cfg, split_reduce_kernel<2>, part, plane, o, vec); break;
    case 4: e = cudaLaunchKernelEx(&cfg, split_reduce_kernel<4>, part, plane, o, vec); break;
    case 8: e = cudaLaunchKernelEx(&cfg, split_reduce_kernel<8>, part, plane, o, vec); break;
    case 16: e = cudaLaunchKernelEx(&cfg, split_reduce_kernel<16>, part, plane, o, vec); break;
    default: return set_error(FL_ERR_ARG, "split reduce: %d slices (2, 4, 8 or 16)", split);
  }
  if (e != cudaSuccess) return set_error(FL_ERR_CUDA, "split reduce launch: %s", cudaGetErrorString(e));
  return FL_OK;
}

}  // namespace fl
