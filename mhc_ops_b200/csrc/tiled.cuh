// Tiled backward for the shapes the tensor-core backward does not take (n other
// than 4: the n = 8 "wide" hyper-connection above all), on the CUDA cores.
//
// Math: src/backward/golden.py:38-96, split as in the tensor-core backward:
//   * rowdot::bwd_rows_kernel<n> leaves one record per token, {dh_mix[N], c,
//     h_pre[n]} (golden.py:49-62, 74, 89), and the dalpha/dbias partials;
//   * dx_kernel: dx[t,k] = (sum_j dh_mix[t,j] phi[j,k]) gamma[k] - c[t] x[t,k]
//     + h_pre[t,i] dh_in[t,d]  (k = i*D + d; golden.py:65, 89-94) -- a
//     [T,N] x [N,nD] product tiled through shared memory, 64 tokens x 128 k
//     per CTA, 8 x 4 outputs per thread, the N-term sum in fp32 FMAs in
//     ascending j (the generic kernel's order);
//   * g_kernel: gpart[p][j][k] = sum over the tokens of split p of
//     dh_mix[t,j] x[t,k] (the un-scaled dphi, golden.py:68-69), 128 k x all N
//     per CTA, 32-token chunks through shared memory, 10 x 4 outputs per
//     thread at n = 8, tokens summed in ascending order;
//   * generic::finalize_param_kernel / reduce_columns_kernel as in the
//     tensor-core backward (fixed order, so results repeat bit for bit).
// Needs D % 8 == 0 and 16-byte aligned x, dh_in, dx and phi.
#pragma once

#include "common.cuh"

namespace mhc {
namespace tiled {

constexpr int kThreads = 256;
constexpr int kTT = 64;    // tokens per dx tile (8 warps x 8 tokens)
constexpr int kKT = 128;   // k per tile (32 lanes x 4 k)
constexpr int kTC = 32;    // tokens per g_kernel chunk

template <int n>
struct Dims {
  static constexpr int N = n * n + 2 * n;
  static constexpr int RW = ((N + 1 + n) + 3) / 4 * 4;   // record width (rowdot::Rec<n>::W)
  static constexpr int JW = (N + 7) / 8;                 // g_kernel: j per warp
  // dx_kernel's dynamic shared memory: dmT [N][kTT], ph [N][kKT], c [kTT], h_pre [kTT][n]
  static constexpr int DX_SMEM = 4 * (N * kTT + N * kKT + kTT + kTT * n);
};

__device__ __forceinline__ void bf16x4(uint2 v, float (&f)[4]) {
  f[0] = __uint_as_float(v.x << 16);
  f[1] = __uint_as_float(v.x & 0xFFFF0000u);
  f[2] = __uint_as_float(v.y << 16);
  f[3] = __uint_as_float(v.y & 0xFFFF0000u);
}

// grid = (ceil(T / kTT), ceil(nD / kKT)), kThreads threads, Dims<n>::DX_SMEM
// bytes of dynamic shared memory.
template <int n>
__global__ void __launch_bounds__(kThreads) dx_kernel(const uint16_t* __restrict__ x, const float* __restrict__ phi,
                                                      const float* __restrict__ gamma, const float* __restrict__ rec,
                                                      const uint16_t* __restrict__ dh_in, uint16_t* __restrict__ dx,
                                                      int64_t T, int D) {
  constexpr int N = Dims<n>::N;
  constexpr int RW = Dims<n>::RW;
  extern __shared__ float4 dx_smem[];
  // dh_mix transposed (a warp's 8 tokens are two float4), phi rows, c, h_pre
  float(*dmT)[kTT] = reinterpret_cast<float(*)[kTT]>(dx_smem);
  float(*ph)[kKT] = reinterpret_cast<float(*)[kKT]>(reinterpret_cast<float*>(dx_smem) + N * kTT);
  float* c_s = reinterpret_cast<float*>(dx_smem) + N * kTT + N * kKT;
  float(*hp_s)[n] = reinterpret_cast<float(*)[n]>(c_s + kTT);
  const int nD = n * D;
  const int64_t t0 = (int64_t)blockIdx.x * kTT;
  const int k0 = blockIdx.y * kKT;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  // records of the tile's tokens (zeros past T)
  for (int e = threadIdx.x; e < kTT * RW; e += kThreads) {
    const int tt = e / RW, c = e - tt * RW;
    const int64_t t = t0 + tt;
    const float v = t < T ? __ldg(rec + t * RW + c) : 0.f;
    if (c < N) dmT[c][tt] = v;
    else if (c == N) c_s[tt] = v;
    else if (c < N + 1 + n) hp_s[tt][c - N - 1] = v;
  }
  // phi rows for the tile's k (zeros past nD)
  for (int e = threadIdx.x; e < N * (kKT / 4); e += kThreads) {
    const int j = e / (kKT / 4), q = e - j * (kKT / 4);
    const int k = k0 + 4 * q;
    const float4 v = k < nD ? __ldg(reinterpret_cast<const float4*>(phi + (int64_t)j * nD + k)) : make_float4(0, 0, 0, 0);
    *reinterpret_cast<float4*>(&ph[j][4 * q]) = v;
  }
  __syncthreads();

  float acc[8][4];
#pragma unroll
  for (int a = 0; a < 8; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
#pragma unroll 4
  for (int j = 0; j < N; ++j) {
    const float4 d0 = *reinterpret_cast<const float4*>(&dmT[j][8 * warp]);
    const float4 d1 = *reinterpret_cast<const float4*>(&dmT[j][8 * warp + 4]);
    const float4 p = *reinterpret_cast<const float4*>(&ph[j][4 * lane]);
    const float dv[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
    const float pv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(dv[a], pv[b], acc[a][b]);
  }

  const int k = k0 + 4 * lane;
  if (k >= nD) return;
  const int i = k / D, d = k - i * D;   // the 4 k share one stream (D % 4 == 0)
  float gm[4] = {1.f, 1.f, 1.f, 1.f};
  if (gamma) {
    const float4 g = __ldg(reinterpret_cast<const float4*>(gamma + k));
    gm[0] = g.x;
    gm[1] = g.y;
    gm[2] = g.z;
    gm[3] = g.w;
  }
#pragma unroll
  for (int a = 0; a < 8; ++a) {
    const int tt = 8 * warp + a;
    const int64_t t = t0 + tt;
    if (t >= T) break;
    float xf[4], gf[4];
    bf16x4(__ldg(reinterpret_cast<const uint2*>(x + t * nD + k)), xf);
    bf16x4(__ldg(reinterpret_cast<const uint2*>(dh_in + t * D + d)), gf);
    const float c = c_s[tt], hp = hp_s[tt][i];
    float v[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) v[b] = acc[a][b] * gm[b] + ((-c) * xf[b] + hp * gf[b]);
    uint2 o;
    o.x = (uint32_t)f32_to_bf16_bits(v[0]) | ((uint32_t)f32_to_bf16_bits(v[1]) << 16);
    o.y = (uint32_t)f32_to_bf16_bits(v[2]) | ((uint32_t)f32_to_bf16_bits(v[3]) << 16);
    *reinterpret_cast<uint2*>(dx + t * nD + k) = o;
  }
}

// grid = (ceil(nD / kKT), P), kThreads threads; split p sums tokens
// [p * per_split, min(T, (p + 1) * per_split)).
template <int n>
__global__ void __launch_bounds__(kThreads) g_kernel(const uint16_t* __restrict__ x, const float* __restrict__ rec,
                                                     float* __restrict__ gpart, int64_t T, int nD, int64_t per_split) {
  constexpr int N = Dims<n>::N;
  constexpr int RW = Dims<n>::RW;
  constexpr int JW = Dims<n>::JW;
  __shared__ __align__(16) float xs[kTC][kKT];
  __shared__ float dm[kTC][8 * JW];
  const int k0 = blockIdx.x * kKT;
  const int p = blockIdx.y;
  const int64_t ta = (int64_t)p * per_split;
  const int64_t tb = min(T, ta + per_split);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float acc[JW][4];
#pragma unroll
  for (int a = 0; a < JW; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;

  for (int64_t tc = ta; tc < tb; tc += kTC) {
    __syncthreads();   // the previous chunk is used up
    // x chunk [kTC tokens][kKT k] as fp32 (zeros past T or nD)
    for (int e = threadIdx.x; e < kTC * (kKT / 8); e += kThreads) {
      const int tt = e / (kKT / 8), q = e - tt * (kKT / 8);
      const int64_t t = tc + tt;
      const int k = k0 + 8 * q;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (t < tb && k < nD) v = __ldg(reinterpret_cast<const uint4*>(x + t * nD + k));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        xs[tt][8 * q + 2 * h] = __uint_as_float(w[h] << 16);
        xs[tt][8 * q + 2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u);
      }
    }
    // dh_mix of the chunk's tokens, j padded to 8 * JW with zeros
    for (int e = threadIdx.x; e < kTC * 8 * JW; e += kThreads) {
      const int tt = e / (8 * JW), j = e - tt * (8 * JW);
      const int64_t t = tc + tt;
      dm[tt][j] = (t < tb && j < N) ? __ldg(rec + t * RW + j) : 0.f;
    }
    __syncthreads();
    const int nt = (int)min((int64_t)kTC, tb - tc);
    for (int tt = 0; tt < nt; ++tt) {
      const float4 xv = *reinterpret_cast<const float4*>(&xs[tt][4 * lane]);
      const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int a = 0; a < JW; ++a) {
        const float dv = dm[tt][warp * JW + a];
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(dv, xa[b], acc[a][b]);
      }
    }
  }
  const int k = k0 + 4 * lane;
  if (k >= nD) return;
#pragma unroll
  for (int a = 0; a < JW; ++a) {
    const int j = warp * JW + a;
    if (j < N)
      *reinterpret_cast<float4*>(gpart + ((int64_t)p * N + j) * nD + k) =
          make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
  }
}

}  // namespace tiled
}  // namespace mhc
