// Shared helpers of libmhc_ops: status handling, bf16 conversion, launch counting.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <atomic>
#include <cstring>

#include "../../include/mhc_ops.h"

namespace mhc {

// Byte layout of the header every workspace starts with.  The device status
// word is written by kernels whose bounded waits expire and read back by
// mhc_read_device_status().
constexpr size_t kWsHeaderBytes = 256;
constexpr size_t kWsAlign = 256;

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

extern std::atomic<uint64_t> g_launch_count;
void set_last_cuda_error(cudaError_t e);

#define MHC_CUDA_TRY(expr)                         \
  do {                                             \
    cudaError_t _e = (expr);                       \
    if (_e != cudaSuccess) {                       \
      ::mhc::set_last_cuda_error(_e);              \
      return MHC_ERR_CUDA;                         \
    }                                              \
  } while (0)

// Call after every kernel launch: counts it and maps launch errors.
inline int after_launch() {
  g_launch_count.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return MHC_ERR_CUDA;
  }
  return MHC_OK;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Round-to-nearest-even float -> bf16 bits (NaN kept quiet), the rounding of
// torch.Tensor.to(torch.bfloat16).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Two floats -> packed bf16x2 bits (lo in the low half), round-to-nearest-even,
// one conversion instruction for both.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + __expf(-v)); }

// Exact-ish sigmoid using the accurate expf (the gates feed fp32 outputs that
// are compared at 1e-4 relative; expf keeps them at ~1e-7).
__device__ __forceinline__ float sigmoid_acc(float v) { return 1.0f / (1.0f + expf(-v)); }

// Warp reduction of one float.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void set_device_status(int* status, int code) {
  if (status != nullptr) atomicExch(status, code);
}

}  // namespace mhc
