// Shared helpers of libmhc_ops: status handling, bf16 conversion, launch counting.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <atomic>
#include <cstring>
#include <type_traits>

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

// t-th bf16 term of v (0 = hi, 1 = mid, 2 = lo): each rounds what is left.
__device__ __forceinline__ uint16_t split_term(float v, int term) {
  uint16_t out = 0;
  for (int tt = 0; tt <= term; ++tt) {
    out = f32_to_bf16_bits(v);
    v -= bf16_bits_to_f32(out);
  }
  return out;
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

// ------------------------------------------------------------------ debug-bounds builds
// Built with -DMHC_DEBUG_BOUNDS (python -m mhc_ops_b200.build --debug-bounds,
// lib/libmhc_ops_dbg.so), every global access written through MHC_CHK /
// MHC_LD / MHC_LDG / MHC_ST / MHC_LDP / MHC_STP is checked against the buffers
// of the current call, which each entry point registers before it launches
// (the argument tensors and the workspace, with their byte sizes).  An access
// that does not lie inside one of them is not made -- nothing traps -- and the
// first one is recorded
// {count, site, address, bytes}; mhc_debug_bounds() returns the record.  The
// site is file id * 100000 + source line.  TMA accesses need no check: the
// tensor maps clip them.  One call at a time per process in these builds (the
// buffer table is global).  In normal builds the macros are the bare access.
constexpr int kDbgBufs = 32;
struct DbgBuf {
  unsigned long long lo, hi;   // [lo, hi) bytes
};
#ifdef MHC_DEBUG_BOUNDS
__device__ DbgBuf g_dbg_bufs[kDbgBufs];
__device__ int g_dbg_nbufs;
__device__ unsigned long long g_dbg_oob[4];
__device__ uint4 g_dbg_zero;   // what a failed checked load reads (never written)
__device__ uint4 g_dbg_sink;   // where a failed checked store goes

__device__ __noinline__ bool dbg_check(const void* p, unsigned bytes, unsigned site) {
  const unsigned long long a = reinterpret_cast<unsigned long long>(p), b = a + bytes;
  const int nb = g_dbg_nbufs;
  for (int i = 0; i < nb && i < kDbgBufs; ++i)
    if (a >= g_dbg_bufs[i].lo && b <= g_dbg_bufs[i].hi) return true;
  if (atomicAdd(&g_dbg_oob[0], 1ull) == 0ull) {
    g_dbg_oob[1] = site;
    g_dbg_oob[2] = a;
    g_dbg_oob[3] = bytes;
  }
  return false;
}
// A failed check redirects the access (loads read zeros, stores land in a
// sink) instead of branching around it, so the arithmetic around a checked
// access compiles as in a normal build (same FMA contractions, same bits).
template <class T>
__device__ __forceinline__ T* dbg_ld_ptr(T* p, unsigned bytes, unsigned site) {
  return dbg_check(p, bytes, site) ? p : reinterpret_cast<T*>(&g_dbg_zero);
}
template <class T>
__device__ __forceinline__ T* dbg_st_ptr(T* p, unsigned bytes, unsigned site) {
  return dbg_check(p, bytes, site) ? p : reinterpret_cast<T*>(&g_dbg_sink);
}
#define MHC_SITE ((unsigned)(MHC_FILE_ID * 100000 + __LINE__))
#define MHC_CHK(p, bytes) ::mhc::dbg_check((p), (unsigned)(bytes), MHC_SITE)
#define MHC_LDP(p, bytes) ::mhc::dbg_ld_ptr((p), (unsigned)(bytes), MHC_SITE)   // at most 16 bytes
#define MHC_STP(p, bytes) ::mhc::dbg_st_ptr((p), (unsigned)(bytes), MHC_SITE)   // at most 16 bytes
#define MHC_LDG(p) __ldg(MHC_LDP((p), sizeof(*(p))))
#define MHC_LD(p) (*MHC_LDP((p), sizeof(*(p))))
#define MHC_ST(p, v) (void)(*MHC_STP((p), sizeof(*(p))) = (v))
#else
#define MHC_CHK(p, bytes) true
#define MHC_LDP(p, bytes) (p)
#define MHC_STP(p, bytes) (p)
#define MHC_LDG(p) __ldg(p)
#define MHC_LD(p) (*(p))
#define MHC_ST(p, v) (void)(*(p) = (v))
#endif
#ifndef MHC_FILE_ID
#define MHC_FILE_ID 0
#endif

}  // namespace mhc
