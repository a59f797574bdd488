// The mHC post-op, the consumer of the pre-op's h_post and h_res: the next
// residual stream of a hyper-connection block,
//   out[t,i,:] = sum_j h_res[t,i,j] x[t,j,:] + h_post[t,i] y[t,:]
// with x [T,n,D] bf16 the block's input streams, y [T,D] bf16 the sublayer's
// output f(h_in), and its backward from dout [T,n,D] bf16:
//   dx[t,j,:]     = sum_i h_res[t,i,j] dout[t,i,:]            (bf16)
//   dy[t,:]       = sum_i h_post[t,i] dout[t,i,:]              (bf16)
//   dh_res[t,i,j] = sum_d dout[t,i,d] x[t,j,d]                 (fp32)
//   dh_post[t,i]  = sum_d dout[t,i,d] y[t,d]                   (fp32)
// The reference (folrent1896/mhc_ops) stops at h_post / h_res
// (src/forward/golden.py:65-69); this is the adjacent step of the block.
//
// Both kernels stream HBM once (x, y read; out written / dout, x, y read;
// dx, dy written).  The bf16 outputs are sums of products in ascending term
// order with every multiply and add rounded on its own (no FMA contraction),
// then one round-to-nearest-even to bf16, so they repeat bit for bit and
// match a float32 restatement of the same order exactly.  The fp32 row sums
// run in a fixed order (each lane's vectors in turn, then a fixed shuffle
// tree), so they repeat bit for bit too.
#pragma once

#include "common.cuh"

#undef MHC_FILE_ID
#define MHC_FILE_ID 3   // debug-bounds site ids: 3 * 100000 + line

namespace mhc {
namespace post {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kU = 4;   // vectors per lane of one forward warp task

// V consecutive bf16 of a row -> float (V = 8: one 16-byte load)
template <int V>
__device__ __forceinline__ void load_bf16(const uint16_t* p, float (&f)[V]) {
  if constexpr (V == 8) {
    const uint4 u = MHC_LDG(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      f[2 * h] = __uint_as_float(w[h] << 16);
      f[2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u);
    }
  } else {
#pragma unroll
    for (int e = 0; e < V; ++e) f[e] = bf16_bits_to_f32(MHC_LDG(p + e));
  }
}

template <int V>
__device__ __forceinline__ void store_bf16(uint16_t* p, const float (&f)[V]) {
  if constexpr (V == 8) {
    MHC_ST(reinterpret_cast<uint4*>(p),
           make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7])));
  } else {
#pragma unroll
    for (int e = 0; e < V; ++e) MHC_ST(p + e, f32_to_bf16_bits(f[e]));
  }
}

// Forward.  A warp task is (token t, a run of 32 * kU vectors of V elements);
// lane l takes the vectors l, l + 32, ... of the run, so every load and store
// instruction of the warp covers 32 consecutive vectors.  Grid-stride over
// the T * ceil(D / V / (32 kU)) tasks, kWarps warps per CTA.
template <int n, int V>
__global__ void __launch_bounds__(kThreads) post_fwd_kernel(const uint16_t* __restrict__ x,
                                                            const float* __restrict__ h_res,
                                                            const float* __restrict__ h_post,
                                                            const uint16_t* __restrict__ y,
                                                            uint16_t* __restrict__ out, int64_t T, int D) {
  const int lane = threadIdx.x & 31;
  const int DV = D / V;
  const int runs = (DV + 32 * kU - 1) / (32 * kU);
  const int64_t tasks = T * runs;
  for (int64_t task = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); task < tasks;
       task += (int64_t)gridDim.x * kWarps) {
    const int64_t t = task / runs;
    const int run = (int)(task - t * runs);
    float cr[n][n], cp[n];
#pragma unroll
    for (int i = 0; i < n; ++i) {
      cp[i] = MHC_LDG(h_post + t * n + i);
#pragma unroll
      for (int j = 0; j < n; ++j) cr[i][j] = MHC_LDG(h_res + (t * n + i) * n + j);
    }
    const uint16_t* xt = x + t * n * D;
    uint16_t* ot = out + t * n * D;
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int v = run * 32 * kU + u * 32 + lane;
      if (v >= DV) break;
      const int d0 = v * V;
      float yv[V], xv[n][V];
      load_bf16<V>(y + t * D + d0, yv);
#pragma unroll
      for (int j = 0; j < n; ++j) load_bf16<V>(xt + (int64_t)j * D + d0, xv[j]);
#pragma unroll
      for (int i = 0; i < n; ++i) {
        float o[V];
#pragma unroll
        for (int e = 0; e < V; ++e) {
          float acc = __fmul_rn(cr[i][0], xv[0][e]);
#pragma unroll
          for (int j = 1; j < n; ++j) acc = __fadd_rn(acc, __fmul_rn(cr[i][j], xv[j][e]));
          o[e] = __fadd_rn(acc, __fmul_rn(cp[i], yv[e]));
        }
        store_bf16<V>(ot + (int64_t)i * D + d0, o);
      }
    }
  }
}

// Backward.  One warp per token (grid-stride over tokens): lane l takes the
// vectors l, l + 32, ... of the row, writes dx and dy for them, and keeps
// running sums of dout[i] . x[j] and dout[i] . y over its vectors; a fixed
// xor-shuffle tree then sums the 32 lanes and lane 0 writes dh_res, dh_post.
template <int n, int V>
__global__ void __launch_bounds__(kThreads, (n <= 4 ? 2 : 1)) post_bwd_kernel(const uint16_t* __restrict__ x,
                                                            const float* __restrict__ h_res,
                                                            const float* __restrict__ h_post,
                                                            const uint16_t* __restrict__ y,
                                                            const uint16_t* __restrict__ dout,
                                                            uint16_t* __restrict__ dx, uint16_t* __restrict__ dy,
                                                            float* __restrict__ dh_res, float* __restrict__ dh_post,
                                                            int64_t T, int D) {
  const int lane = threadIdx.x & 31;
  const int DV = D / V;
  for (int64_t t = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); t < T; t += (int64_t)gridDim.x * kWarps) {
    float cr[n][n], cp[n];
#pragma unroll
    for (int i = 0; i < n; ++i) {
      cp[i] = MHC_LDG(h_post + t * n + i);
#pragma unroll
      for (int j = 0; j < n; ++j) cr[i][j] = MHC_LDG(h_res + (t * n + i) * n + j);
    }
    float sr[n][n], sp[n];
#pragma unroll
    for (int i = 0; i < n; ++i) {
      sp[i] = 0.f;
#pragma unroll
      for (int j = 0; j < n; ++j) sr[i][j] = 0.f;
    }
    const uint16_t* xt = x + t * n * D;
    const uint16_t* gt = dout + t * n * D;
    uint16_t* dxt = dx + t * n * D;
    for (int v = lane; v < DV; v += 32) {
      const int d0 = v * V;
      float g[n][V], yv[V];
#pragma unroll
      for (int i = 0; i < n; ++i) load_bf16<V>(gt + (int64_t)i * D + d0, g[i]);
      load_bf16<V>(y + t * D + d0, yv);
      {
        float o[V];
#pragma unroll
        for (int e = 0; e < V; ++e) {
          float acc = __fmul_rn(cp[0], g[0][e]);
#pragma unroll
          for (int i = 1; i < n; ++i) acc = __fadd_rn(acc, __fmul_rn(cp[i], g[i][e]));
          o[e] = acc;
        }
        store_bf16<V>(dy + t * D + d0, o);
      }
#pragma unroll
      for (int i = 0; i < n; ++i)
#pragma unroll
        for (int e = 0; e < V; ++e) sp[i] = fmaf(g[i][e], yv[e], sp[i]);
#pragma unroll
      for (int j = 0; j < n; ++j) {
        float xv[V], o[V];
        load_bf16<V>(xt + (int64_t)j * D + d0, xv);
#pragma unroll
        for (int e = 0; e < V; ++e) {
          float acc = __fmul_rn(cr[0][j], g[0][e]);
#pragma unroll
          for (int i = 1; i < n; ++i) acc = __fadd_rn(acc, __fmul_rn(cr[i][j], g[i][e]));
          o[e] = acc;
        }
        store_bf16<V>(dxt + (int64_t)j * D + d0, o);
#pragma unroll
        for (int i = 0; i < n; ++i)
#pragma unroll
          for (int e = 0; e < V; ++e) sr[i][j] = fmaf(g[i][e], xv[e], sr[i][j]);
      }
    }
#pragma unroll
    for (int i = 0; i < n; ++i) {
      sp[i] = warp_sum(sp[i]);
#pragma unroll
      for (int j = 0; j < n; ++j) sr[i][j] = warp_sum(sr[i][j]);
    }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < n; ++i) {
        MHC_ST(dh_post + t * n + i, sp[i]);
#pragma unroll
        for (int j = 0; j < n; ++j) MHC_ST(dh_res + (t * n + i) * n + j, sr[i][j]);
      }
    }
  }
}

}  // namespace post
}  // namespace mhc
