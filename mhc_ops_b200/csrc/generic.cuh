// Generic-shape CUDA kernels of the mHC pre-op (any n in [1,8], any D).
//
// These run every shape the tensor-core kernels do not take (D not a multiple
// of 64, tiny token counts, odd n).  One CTA walks one token at a time; the
// projection re-reads phi from L2 per token, so they are correct but far from
// the HBM roofline.  The parameter-gradient reduction (bwd_g / finalize) is
// shared with the tensor-core backward.
#pragma once

#include "common.cuh"

#undef MHC_FILE_ID
#define MHC_FILE_ID 1   // debug-bounds site ids: 1 * 100000 + line

namespace mhc {
namespace generic {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

template <int n>
struct Dims {
  static constexpr int N = n * n + 2 * n;
};

// Sum NV per-thread values over the CTA; every thread gets the totals in out[].
// red must hold kWarps * NV floats.  Order is fixed (deterministic).
template <int NV>
__device__ __forceinline__ void block_sum(float (&v)[NV], float* red, float* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < NV; ++j) v[j] = warp_sum(v[j]);
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < NV; ++j) red[warp * NV + j] = v[j];
  }
  __syncthreads();
  for (int j = threadIdx.x; j < NV; j += kThreads) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[w * NV + j];
    out[j] = s;
  }
  __syncthreads();
}

// Forward, one token per CTA iteration (golden.py:34-69).
template <int n>
__global__ void __launch_bounds__(kThreads) fwd_kernel(
    const uint16_t* __restrict__ x, const float* __restrict__ phi, const float* __restrict__ alpha,
    const float* __restrict__ bias, uint16_t* __restrict__ h_in, float* __restrict__ h_post,
    float* __restrict__ h_res, float* __restrict__ inv_rms_out, float* __restrict__ h_mix_out,
    float* __restrict__ h_pre_out, int64_t T, int D, float norm_eps, float hc_eps,
    float* __restrict__ h_in_rstd = nullptr, float h_in_eps = 0.f) {
  constexpr int N = Dims<n>::N;
  const int nD = n * D;
  __shared__ float red[kWarps * (N + 1)];
  __shared__ float tot[N + 1];
  __shared__ float hpre_s[n];

  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const uint16_t* xr = x + t * (int64_t)nD;
    float acc[N + 1];
#pragma unroll
    for (int j = 0; j <= N; ++j) acc[j] = 0.f;
    for (int k = threadIdx.x; k < nD; k += kThreads) {
      const float xv = bf16_bits_to_f32(MHC_LD(&xr[k]));
      acc[N] = fmaf(xv, xv, acc[N]);
#pragma unroll
      for (int j = 0; j < N; ++j) acc[j] = fmaf(xv, MHC_LDG(phi + (int64_t)j * nD + k), acc[j]);
    }
    block_sum<N + 1>(acc, red, tot);

    if (threadIdx.x == 0) {
      const float ir = 1.0f / sqrtf(tot[N] / (float)nD + norm_eps);
      const float a_pre = MHC_LD(&alpha[0]), a_post = MHC_LD(&alpha[1]), a_res = MHC_LD(&alpha[2]);
      if (inv_rms_out) MHC_ST(&inv_rms_out[t], ir);
      for (int j = 0; j < N; ++j)
        if (h_mix_out) MHC_ST(&h_mix_out[t * N + j], tot[j]);
      for (int i = 0; i < n; ++i) {
        const float hp = sigmoid_acc(a_pre * (tot[i] * ir) + MHC_LD(&bias[i])) + hc_eps;
        hpre_s[i] = hp;
        if (h_pre_out) MHC_ST(&h_pre_out[t * n + i], hp);
        MHC_ST(&h_post[t * n + i], 2.0f * sigmoid_acc(a_post * (tot[n + i] * ir) + MHC_LD(&bias[n + i])));
      }
      for (int m = 0; m < n * n; ++m) MHC_ST(&h_res[t * n * n + m], a_res * (tot[2 * n + m] * ir) + MHC_LD(&bias[2 * n + m]));
    }
    __syncthreads();
    float sq[1] = {0.f};   // sum of the bf16 h_in values squared (h_in_rstd)
    for (int d = threadIdx.x; d < D; d += kThreads) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < n; ++i) s = fmaf(hpre_s[i], bf16_bits_to_f32(MHC_LD(&xr[i * D + d])), s);
      const uint16_t b = f32_to_bf16_bits(s);
      MHC_ST(&h_in[t * D + d], b);
      const float r = bf16_bits_to_f32(b);
      sq[0] = fmaf(r, r, sq[0]);
    }
    __syncthreads();
    if (h_in_rstd) {
      block_sum<1>(sq, red, tot);
      if (threadIdx.x == 0) MHC_ST(&h_in_rstd[t], 1.0f / sqrtf(tot[0] / (float)D + h_in_eps));
      __syncthreads();
    }
  }
}

// Backward, per-token part (src/backward/golden.py:49-62, 72-94): dx, plus
// dh_mix [T,N] and the per-token dalpha/dbias terms [T,3+N] for the
// fixed-order reductions that follow.
template <int n>
__global__ void __launch_bounds__(kThreads) bwd_token_kernel(
    const uint16_t* __restrict__ x, const float* __restrict__ phi, const float* __restrict__ alpha,
    const float* __restrict__ inv_rms, const float* __restrict__ h_mix, const float* __restrict__ h_pre,
    const float* __restrict__ h_post, const uint16_t* __restrict__ dh_in,
    const float* __restrict__ dh_post, const float* __restrict__ dh_res, const float* __restrict__ gamma,
    uint16_t* __restrict__ dx, float* __restrict__ dh_mix_ws, float* __restrict__ tokpart, int64_t T,
    int D, float hc_eps) {
  constexpr int N = Dims<n>::N;
  constexpr int W = 3 + N;
  const int nD = n * D;
  __shared__ float red[kWarps * n];
  __shared__ float tot[n];
  __shared__ float dmix_s[N];
  __shared__ float hpre_s[n];
  __shared__ float c_s;

  for (int64_t t = blockIdx.x; t < T; t += gridDim.x) {
    const uint16_t* xr = x + t * (int64_t)nD;
    const uint16_t* gr = dh_in + t * (int64_t)D;
    float p[n];
#pragma unroll
    for (int i = 0; i < n; ++i) p[i] = 0.f;
    for (int d = threadIdx.x; d < D; d += kThreads) {
      const float g = bf16_bits_to_f32(MHC_LD(&gr[d]));
#pragma unroll
      for (int i = 0; i < n; ++i) p[i] = fmaf(g, bf16_bits_to_f32(MHC_LD(&xr[i * D + d])), p[i]);
    }
    block_sum<n>(p, red, tot);

    if (threadIdx.x == 0) {
      const float a_pre = MHC_LD(&alpha[0]), a_post = MHC_LD(&alpha[1]), a_res = MHC_LD(&alpha[2]);
      const float ir = MHC_LD(&inv_rms[t]);
      float tmp[N];
      float dal0 = 0.f, dal1 = 0.f, dal2 = 0.f, dinv = 0.f;
      float* tp = tokpart + t * W;
      for (int i = 0; i < n; ++i) {
        const float hp = MHC_LD(&h_pre[t * n + i]);
        hpre_s[i] = hp;
        const float s = hp - hc_eps;
        const float dpre2 = tot[i] * s * (1.0f - s);
        const float hq = MHC_LD(&h_post[t * n + i]);
        const float dpost2 = MHC_LD(&dh_post[t * n + i]) * hq * (1.0f - hq / 2.0f);
        tmp[i] = a_pre * dpre2;
        tmp[n + i] = a_post * dpost2;
        dal0 += dpre2 * (MHC_LD(&h_mix[t * N + i]) * ir);
        dal1 += dpost2 * (MHC_LD(&h_mix[t * N + n + i]) * ir);
        MHC_ST(&tp[3 + i], dpre2);
        MHC_ST(&tp[3 + n + i], dpost2);
      }
      for (int m = 0; m < n * n; ++m) {
        const float dr = MHC_LD(&dh_res[t * n * n + m]);
        tmp[2 * n + m] = a_res * dr;
        dal2 += dr * (MHC_LD(&h_mix[t * N + 2 * n + m]) * ir);
        MHC_ST(&tp[3 + 2 * n + m], dr);
      }
      for (int j = 0; j < N; ++j) {
        dinv += tmp[j] * MHC_LD(&h_mix[t * N + j]);
        const float dm = tmp[j] * ir;
        dmix_s[j] = dm;
        MHC_ST(&dh_mix_ws[t * N + j], dm);
      }
      MHC_ST(&tp[0], dal0);
      MHC_ST(&tp[1], dal1);
      MHC_ST(&tp[2], dal2);
      c_s = dinv * (ir * ir * ir) / (float)nD;
    }
    __syncthreads();
    const float c = c_s;
    for (int k = threadIdx.x; k < nD; k += kThreads) {
      const int i = k / D, d = k - i * D;
      float mm = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) mm = fmaf(dmix_s[j], MHC_LDG(phi + (int64_t)j * nD + k), mm);
      const float gmm = gamma ? MHC_LD(&gamma[k]) : 1.0f;
      const float v = mm * gmm + ((-c) * bf16_bits_to_f32(MHC_LD(&xr[k])) + hpre_s[i] * bf16_bits_to_f32(MHC_LD(&gr[d])));
      MHC_ST(&dx[t * (int64_t)nD + k], f32_to_bf16_bits(v));
    }
    __syncthreads();
  }
}

// G partials: gpart[p][j][k] = sum over tokens of split p of dh_mix[t][j] * x[t][k]
// (the un-scaled dphi of golden.py:68-69).  grid = (ceil(nD/256), P).
template <int n>
__global__ void __launch_bounds__(kThreads) bwd_g_kernel(const uint16_t* __restrict__ x,
                                                         const float* __restrict__ dh_mix_ws,
                                                         float* __restrict__ gpart, int64_t T, int nD,
                                                         int64_t tokens_per_split) {
  constexpr int N = Dims<n>::N;
  const int k = blockIdx.x * kThreads + threadIdx.x;
  const int p = blockIdx.y;
  const int64_t t0 = (int64_t)p * tokens_per_split;
  const int64_t t1 = min(T, t0 + tokens_per_split);
  float acc[N];
#pragma unroll
  for (int j = 0; j < N; ++j) acc[j] = 0.f;
  if (k < nD) {
    for (int64_t t = t0; t < t1; ++t) {
      const float xv = bf16_bits_to_f32(MHC_LD(&x[t * nD + k]));
#pragma unroll
      for (int j = 0; j < N; ++j) acc[j] = fmaf(MHC_LDG(dh_mix_ws + t * N + j), xv, acc[j]);
    }
#pragma unroll
    for (int j = 0; j < N; ++j) MHC_ST(&gpart[((int64_t)p * N + j) * nD + k], acc[j]);
  }
}

// dalpha / dbias: column c of part [rows][W] summed over rows in a fixed
// order (thread r takes rows r, r + kThreads, ...; then warps, then the 8
// warp sums in order); c < 3 -> dalpha[c], else dbias[c - 3].
__device__ __forceinline__ void reduce_column(const float* __restrict__ part, int64_t rows, int W, int c,
                                              float* __restrict__ dalpha, float* __restrict__ dbias) {
  __shared__ float red[kWarps];
  float s = 0.f;
#pragma unroll 4
  for (int64_t r = threadIdx.x; r < rows; r += kThreads) s += MHC_LD(&part[r * W + c]);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < kWarps; ++w) tot += red[w];
    if (c < 3) MHC_ST(&dalpha[c], tot);
    else MHC_ST(&dbias[c - 3], tot);
  }
}

// dphi[j][k] = gamma[k] * sum_p gpart[p][j][k]; dgamma[k] = sum_j phi[j][k] * G[j][k].
// CTA = 32 columns k x 8 row groups (j = jg, jg+8, ...); the 8 dgamma partials
// are added in a fixed order.  Launch with ceil(nD / kFinCols) + 3 + N CTAs of
// kThreads: the trailing 3 + N CTAs sum the dalpha / dbias columns of abpart
// [ab_rows][3 + N] (reduce_column).
constexpr int kFinCols = 32;
template <int N>
__global__ void __launch_bounds__(kThreads) finalize_param_kernel(const float* __restrict__ gpart, int P,
                                                                  const float* __restrict__ phi,
                                                                  const float* __restrict__ gamma,
                                                                  float* __restrict__ dphi,
                                                                  float* __restrict__ dgamma, int nD,
                                                                  const float* __restrict__ abpart, int64_t ab_rows,
                                                                  float* __restrict__ dalpha,
                                                                  float* __restrict__ dbias) {
  const int kblocks = (nD + kFinCols - 1) / kFinCols;
  if ((int)blockIdx.x >= kblocks) {   // the 3 + N trailing CTAs: dalpha / dbias columns
    reduce_column(abpart, ab_rows, 3 + N, (int)blockIdx.x - kblocks, dalpha, dbias);
    return;
  }
  constexpr int JG = kThreads / kFinCols;
  constexpr int JPER = (N + JG - 1) / JG;   // j = jg, jg + JG, ... of this thread
  __shared__ float part[JG][kFinCols];
  const int kk = threadIdx.x % kFinCols, jg = threadIdx.x / kFinCols;
  const int k = blockIdx.x * kFinCols + kk;
  float dg = 0.f;
  if (k < nD) {
    const float gm = gamma ? MHC_LDG(gamma + k) : 1.0f;
    // splits outer, this thread's rows inner: JPER independent loads per step,
    // each row still summed over p in ascending order
    float g[JPER];
#pragma unroll
    for (int q = 0; q < JPER; ++q) g[q] = 0.f;
    for (int p = 0; p < P; ++p) {
#pragma unroll
      for (int q = 0; q < JPER; ++q) {
        const int j = jg + q * JG;
        if (j < N) g[q] += MHC_LDG(gpart + ((int64_t)p * N + j) * nD + k);
      }
    }
#pragma unroll
    for (int q = 0; q < JPER; ++q) {
      const int j = jg + q * JG;
      if (j < N) {
        MHC_ST(&dphi[(int64_t)j * nD + k], gm * g[q]);
        dg = fmaf(MHC_LDG(phi + (int64_t)j * nD + k), g[q], dg);
      }
    }
  }
  part[jg][kk] = dg;
  __syncthreads();
  if (jg == 0 && k < nD) {
    float s = part[0][kk];
#pragma unroll
    for (int g2 = 1; g2 < JG; ++g2) s += part[g2][kk];
    MHC_ST(&dgamma[k], s);
  }
}

}  // namespace generic
}  // namespace mhc
