// Tiled backward for the shapes the tensor-core backward does not take (n other
// than 4: the n = 8 "wide" hyper-connection above all), on the CUDA cores.
//
// Math: src/backward/golden.py:38-96, split as in the tensor-core backward:
//   * rowdot::bwd_rows_kernel<n> leaves one record per token, {dh_mix[N], c,
//     h_pre[n]} (golden.py:49-62, 74, 89), and the dalpha/dbias partials;
//   * transpose_kernel turns the records' dh_mix into dmT [N][Tp] (token
//     fastest), the layout the dx tiles read;
//   * dx_kernel: dx[t,k] = (sum_j dh_mix[t,j] phi[j,k]) gamma[k] - c[t] x[t,k]
//     + h_pre[t,i] dh_in[t,d]  (k = i*D + d; golden.py:65, 89-94) -- a
//     [T,N] x [N,nD] product tiled through shared memory (cp.async), 64
//     tokens x 256 k per CTA, 8 x 8 outputs per thread, the N-term sum in
//     fp32 FMAs in ascending j (the generic kernel's order);
//   * g_kernel: gpart[p][j][k] = sum over the tokens of split p of
//     dh_mix[t,j] x[t,k] (the un-scaled dphi, golden.py:68-69), 256 k x all N
//     per CTA, 16-token chunks double-buffered through shared memory with
//     cp.async, tokens summed in ascending order;
//   * generic::finalize_param_kernel (dphi, dgamma and the dalpha / dbias
//     column sums) as in the tensor-core backward (fixed order, so results
//     repeat bit for bit).
// Needs D % 8 == 0 and 16-byte aligned x, dh_in, dx, phi and gamma.
#pragma once

#include "common.cuh"

namespace mhc {
namespace tiled {

constexpr int kThreads = 256;
constexpr int kTT = 64;    // tokens per dx tile (8 warps x 8 tokens)
constexpr int kKL = 8;     // consecutive k per lane (one 16-byte bf16 load)
constexpr int kKT = 32 * kKL;   // k per tile
constexpr int kTC = 16;    // tokens per g_kernel chunk

template <int n>
struct Dims {
  static constexpr int N = n * n + 2 * n;
  static constexpr int N4 = (N + 3) / 4 * 4;             // dh_mix floats copied per record (16-byte pieces)
  static constexpr int RW = ((N + 1 + n) + 3) / 4 * 4;   // record width (rowdot::Rec<n>::W)
  static constexpr int JW = (N + 7) / 8;                 // g_kernel: j per warp
  // dx_kernel's dynamic shared memory: dmT [N][kTT], ph [N][kKT], c [kTT], h_pre [kTT][n]
  static constexpr int DX_SMEM = 4 * (N * kTT + N * kKT + kTT + kTT * n);
  static_assert(N4 <= RW && N4 <= 8 * JW, "record copy stays inside the record and the chunk row");
};

// Tokens of the transposed dh_mix (a whole number of dx tiles).
inline int64_t padded_tokens(int64_t T) { return (T + kTT - 1) / kTT * kTT; }

__device__ __forceinline__ void cp16(void* dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst_smem)),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int kPending>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

__device__ __forceinline__ void bf16x4(uint2 v, float (&f)[4]) {
  f[0] = __uint_as_float(v.x << 16);
  f[1] = __uint_as_float(v.x & 0xFFFF0000u);
  f[2] = __uint_as_float(v.y << 16);
  f[3] = __uint_as_float(v.y & 0xFFFF0000u);
}

// rec [T][RW] -> dmT [N][Tp], zeros for tokens T..Tp-1.  grid = (Tp / 32,
// ceil(N / 32)), 256 threads; a 32 x 32 tile through padded shared memory.
template <int n>
__global__ void __launch_bounds__(kThreads) transpose_kernel(const float* __restrict__ rec, float* __restrict__ dmT,
                                                             int64_t T, int64_t Tp) {
  constexpr int N = Dims<n>::N;
  constexpr int RW = Dims<n>::RW;
  __shared__ float tile[32][33];
  const int64_t t0 = (int64_t)blockIdx.x * 32;
  const int j0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int r = ty; r < 32; r += kThreads / 32) {
    const int64_t t = t0 + r;
    const int j = j0 + tx;
    tile[r][tx] = (t < T && j < N) ? __ldg(rec + t * RW + j) : 0.f;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += kThreads / 32) {
    const int j = j0 + r;
    const int64_t t = t0 + tx;
    if (j < N && t < Tp) dmT[(int64_t)j * Tp + t] = tile[tx][r];
  }
}

// grid = (Tp / kTT, ceil(nD / kKT)), kThreads threads, Dims<n>::DX_SMEM bytes
// of dynamic shared memory.
template <int n>
__global__ void __launch_bounds__(kThreads) dx_kernel(const uint16_t* __restrict__ x, const float* __restrict__ phi,
                                                      const float* __restrict__ gamma, const float* __restrict__ rec,
                                                      const float* __restrict__ dmT_g, const uint16_t* __restrict__ dh_in,
                                                      uint16_t* __restrict__ dx, int64_t T, int64_t Tp, int D) {
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

  // dh_mix rows of the tile (Tp covers every tile) and phi rows (zeros past nD)
  for (int e = threadIdx.x; e < N * (kTT / 4); e += kThreads) {
    const int j = e / (kTT / 4), q = e - j * (kTT / 4);
    cp16(&dmT[j][4 * q], dmT_g + (int64_t)j * Tp + t0 + 4 * q);
  }
  for (int e = threadIdx.x; e < N * (kKT / 4); e += kThreads) {
    const int j = e / (kKT / 4), q = e - j * (kKT / 4);
    const int k = k0 + 4 * q;
    if (k < nD) cp16(&ph[j][4 * q], phi + (int64_t)j * nD + k);
    else *reinterpret_cast<float4*>(&ph[j][4 * q]) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  cp_commit();
  for (int e = threadIdx.x; e < kTT * (1 + n); e += kThreads) {
    const int tt = e / (1 + n), c = e - tt * (1 + n);
    const int64_t t = t0 + tt;
    const float v = t < T ? __ldg(rec + t * RW + N + c) : 0.f;
    if (c == 0) c_s[tt] = v;
    else hp_s[tt][c - 1] = v;
  }
  cp_wait<0>();
  __syncthreads();

  // acc2[a][h] holds outputs (token a, k 2h and 2h+1 of the lane's 8);
  // __ffma2_rn rounds each half exactly as fmaf does, two FMAs per instruction
  float2 acc2[8][kKL / 2];
#pragma unroll
  for (int a = 0; a < 8; ++a)
#pragma unroll
    for (int h = 0; h < kKL / 2; ++h) acc2[a][h] = make_float2(0.f, 0.f);
#pragma unroll 2
  for (int j = 0; j < N; ++j) {
    const float4 d0 = *reinterpret_cast<const float4*>(&dmT[j][8 * warp]);
    const float4 d1 = *reinterpret_cast<const float4*>(&dmT[j][8 * warp + 4]);
    const float4 pa = *reinterpret_cast<const float4*>(&ph[j][kKL * lane]);
    const float4 pb = *reinterpret_cast<const float4*>(&ph[j][kKL * lane + 4]);
    const float dv[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
    const float2 pv[kKL / 2] = {make_float2(pa.x, pa.y), make_float2(pa.z, pa.w), make_float2(pb.x, pb.y),
                                make_float2(pb.z, pb.w)};
#pragma unroll
    for (int a = 0; a < 8; ++a) {
      const float2 dd = make_float2(dv[a], dv[a]);
#pragma unroll
      for (int h = 0; h < kKL / 2; ++h) acc2[a][h] = __ffma2_rn(dd, pv[h], acc2[a][h]);
    }
  }

  const int k = k0 + kKL * lane;
  if (k >= nD) return;
  const int i = k / D, d = k - i * D;   // the 8 k share one stream (D % 8 == 0)
  float gm[kKL];
#pragma unroll
  for (int b = 0; b < kKL; ++b) gm[b] = 1.f;
  if (gamma) {
    const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + k));
    const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + k + 4));
    gm[0] = g0.x;
    gm[1] = g0.y;
    gm[2] = g0.z;
    gm[3] = g0.w;
    gm[4] = g1.x;
    gm[5] = g1.y;
    gm[6] = g1.z;
    gm[7] = g1.w;
  }
#pragma unroll
  for (int a = 0; a < 8; ++a) {
    const int tt = 8 * warp + a;
    const int64_t t = t0 + tt;
    if (t >= T) break;
    const uint4 xr = __ldg(reinterpret_cast<const uint4*>(x + t * nD + k));
    const uint4 gr = __ldg(reinterpret_cast<const uint4*>(dh_in + t * D + d));
    float xf[kKL], gf[kKL];
    bf16x4(make_uint2(xr.x, xr.y), *reinterpret_cast<float(*)[4]>(&xf[0]));
    bf16x4(make_uint2(xr.z, xr.w), *reinterpret_cast<float(*)[4]>(&xf[4]));
    bf16x4(make_uint2(gr.x, gr.y), *reinterpret_cast<float(*)[4]>(&gf[0]));
    bf16x4(make_uint2(gr.z, gr.w), *reinterpret_cast<float(*)[4]>(&gf[4]));
    const float c = c_s[tt], hp = hp_s[tt][i];
    uint32_t w[kKL / 2];
#pragma unroll
    for (int h = 0; h < kKL / 2; ++h) {
      const float v0 = acc2[a][h].x * gm[2 * h] + ((-c) * xf[2 * h] + hp * gf[2 * h]);
      const float v1 = acc2[a][h].y * gm[2 * h + 1] + ((-c) * xf[2 * h + 1] + hp * gf[2 * h + 1]);
      w[h] = (uint32_t)f32_to_bf16_bits(v0) | ((uint32_t)f32_to_bf16_bits(v1) << 16);
    }
    *reinterpret_cast<uint4*>(dx + t * nD + k) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// grid = (ceil(nD / kKT), P), kThreads threads; split p sums tokens
// [p * per_split, min(T, (p + 1) * per_split)).
template <int n>
__global__ void __launch_bounds__(kThreads) g_kernel(const uint16_t* __restrict__ x, const float* __restrict__ rec,
                                                     float* __restrict__ gpart, int64_t T, int nD, int64_t per_split) {
  constexpr int N = Dims<n>::N;
  constexpr int N4 = Dims<n>::N4;
  constexpr int RW = Dims<n>::RW;
  constexpr int JW = Dims<n>::JW;
  __shared__ __align__(16) uint16_t xs[2][kTC][kKT];   // raw bf16 chunks
  __shared__ __align__(16) float dm[2][kTC][8 * JW];
  const int k0 = blockIdx.x * kKT;
  const int p = blockIdx.y;
  const int64_t ta = (int64_t)p * per_split;
  const int64_t tb = min(T, ta + per_split);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float2 acc2[JW][kKL / 2];   // (j, k pair): __ffma2_rn, two exact fmaf per instruction
#pragma unroll
  for (int a = 0; a < JW; ++a)
#pragma unroll
    for (int h = 0; h < kKL / 2; ++h) acc2[a][h] = make_float2(0.f, 0.f);

  // chunk tokens [tc, tc + kTC) into buffer b; x columns past nD and tokens
  // past tb are not copied (their products are never summed or stored)
  auto load = [&](int64_t tc, int b) {
    for (int e = threadIdx.x; e < kTC * (kKT / 8); e += kThreads) {
      const int tt = e / (kKT / 8), q = e - tt * (kKT / 8);
      const int64_t t = tc + tt;
      const int k = k0 + 8 * q;
      if (t < tb && k < nD) cp16(&xs[b][tt][8 * q], x + t * nD + k);
    }
    for (int e = threadIdx.x; e < kTC * (N4 / 4); e += kThreads) {
      const int tt = e / (N4 / 4), q = e - tt * (N4 / 4);
      const int64_t t = tc + tt;
      if (t < tb) cp16(&dm[b][tt][4 * q], rec + t * RW + 4 * q);
    }
    cp_commit();
  };

  if (ta < tb) load(ta, 0);
  int b = 0;
  for (int64_t tc = ta; tc < tb; tc += kTC, b ^= 1) {
    const bool more = tc + kTC < tb;
    if (more) {
      load(tc + kTC, b ^ 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();   // chunk tc is in buffer b for every thread
    const int nt = (int)min((int64_t)kTC, tb - tc);
    for (int tt = 0; tt < nt; ++tt) {
      const uint4 xr = *reinterpret_cast<const uint4*>(&xs[b][tt][kKL * lane]);
      float xa[kKL];
      bf16x4(make_uint2(xr.x, xr.y), *reinterpret_cast<float(*)[4]>(&xa[0]));
      bf16x4(make_uint2(xr.z, xr.w), *reinterpret_cast<float(*)[4]>(&xa[4]));
      float2 xv[kKL / 2];
#pragma unroll
      for (int h = 0; h < kKL / 2; ++h) xv[h] = make_float2(xa[2 * h], xa[2 * h + 1]);
      float dv[JW];   // this warp's JW values of dh_mix: float2 broadcasts when JW is even
      if constexpr (JW % 2 == 0) {
#pragma unroll
        for (int a = 0; a < JW; a += 2) {
          const float2 v2 = *reinterpret_cast<const float2*>(&dm[b][tt][warp * JW + a]);
          dv[a] = v2.x;
          dv[a + 1] = v2.y;
        }
      } else {
#pragma unroll
        for (int a = 0; a < JW; ++a) dv[a] = dm[b][tt][warp * JW + a];
      }
#pragma unroll
      for (int a = 0; a < JW; ++a) {
        const float2 dd = make_float2(dv[a], dv[a]);
#pragma unroll
        for (int h = 0; h < kKL / 2; ++h) acc2[a][h] = __ffma2_rn(dd, xv[h], acc2[a][h]);
      }
    }
    __syncthreads();   // buffer b is used up before the next chunk refills it
  }
  const int k = k0 + kKL * lane;
  if (k >= nD) return;
#pragma unroll
  for (int a = 0; a < JW; ++a) {
    const int j = warp * JW + a;
    if (j < N) {
      float4* o = reinterpret_cast<float4*>(gpart + ((int64_t)p * N + j) * nD + k);
      o[0] = make_float4(acc2[a][0].x, acc2[a][0].y, acc2[a][1].x, acc2[a][1].y);
      o[1] = make_float4(acc2[a][2].x, acc2[a][2].y, acc2[a][3].x, acc2[a][3].y);
    }
  }
}

}  // namespace tiled
}  // namespace mhc
