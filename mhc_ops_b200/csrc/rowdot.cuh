// Streaming per-token kernels of the mHC pre-op that need whole token rows
// and no tensor cores: the first kernel of the backward (bwd_rows_kernel) and
// the second kernel of the forward (fwd_rows_kernel).  Pure HBM streams: warps own whole tokens, every load
// is 512 contiguous bytes per warp, many loads in flight per lane.
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "common.cuh"

#undef MHC_FILE_ID
#define MHC_FILE_ID 2   // debug-bounds site ids: 2 * 100000 + line

namespace mhc {
namespace rowdot {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;

template <int n>
struct Rec {
  static constexpr int N_OUT = n * n + 2 * n;
  static constexpr int W = ((N_OUT + 1 + n) + 3) / 4 * 4;   // record width in floats
  static constexpr int CW = 3 + N_OUT;                       // dalpha / dbias columns
};

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  p = MHC_LDP(p, 16);
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void bf16x8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Running dalpha / dbias sums of the tokens one warp has processed.
template <int n>
struct RowAcc {
  static constexpr int N_OUT = Rec<n>::N_OUT;
  static constexpr int M = (N_OUT + 31) / 32;   // output columns per lane
  float al0 = 0.f, al1 = 0.f, al2 = 0.f;        // lane 0
  float b[M];                                   // lane l: dbias[l + 32 m]
  __device__ __forceinline__ RowAcc() {
#pragma unroll
    for (int m = 0; m < M; ++m) b[m] = 0.f;
  }
  // this warp's partial row abpart[CW]: dalpha (3), then dbias (N_OUT)
  __device__ __forceinline__ void store(float* ap, int lane) const {
    if (lane == 0) {
      MHC_ST(ap + 0, al0);
      MHC_ST(ap + 1, al1);
      MHC_ST(ap + 2, al2);
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int jj = lane + 32 * m;
      if (jj < N_OUT) MHC_ST(ap + 3 + jj, b[m]);
    }
  }
};

struct BwdRowArgs {
  const uint16_t* x;
  const uint16_t* dh_in;
  const float* alpha;
  const float* inv_rms;
  const float* h_mix;
  const float* h_pre;
  const float* h_post;
  const float* dh_post;
  const float* dh_res;
  float* rec;
  int D;
  float hc_eps;
  // optional: the split phi * gamma images the next kernel reads (NULL: none)
  const float* img_phi;
  const float* img_gamma;   // NULL = ones
  uint8_t* img;
  int img_blocks;           // 64-k blocks, n*D/64
};

// The split image of phi * gamma for the 64-k block blk, built by one warp:
// row kk (k = 64 blk + kk), column e*SEGW + j = bf16 term e (hi, mid, lo) of
// phi[j][k] * gamma[k] (zeros for j >= N_OUT), K-major interleaved in 8 x
// 16-byte core matrices -- the 16 bytes of (kk, column chunk cc) at
// (kk / 8) * RG + cc * 128 + (kk % 8) * 16, RG = (3 SEGW / 8) * 128 -- as the
// n = 4 tensor-core backward (its phi images) and the tiled dx kernels read
// it.  Lane l builds rows l and l + 32 from its own loads (coalesced across
// the lanes).  Needs n*D % 64 == 0.
template <int n>
__device__ __forceinline__ void split_image_block(const BwdRowArgs& a, int blk, int lane) {
  constexpr int N_OUT = n * n + 2 * n;
  constexpr int SEGW = (N_OUT + 15) / 16 * 16;
  constexpr int CPR = 3 * SEGW / 8;   // 16-byte chunks per image row
  constexpr int RG = CPR * 128;
  const int64_t nD = (int64_t)n * a.D;
  uint8_t* out = a.img + (size_t)blk * 8 * RG;
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    const int kk = lane + 32 * half;
    const int64_t k = (int64_t)blk * 64 + kk;
    const float gm = a.img_gamma ? MHC_LDG(a.img_gamma + k) : 1.0f;
    float v[N_OUT];
#pragma unroll
    for (int j = 0; j < N_OUT; ++j) v[j] = MHC_LDG(a.img_phi + (int64_t)j * nD + k) * gm;
    uint8_t* row = out + (kk >> 3) * RG + (kk & 7) * 16;
#pragma unroll
    for (int cc = 0; cc < CPR; ++cc) {
      const int e = (cc * 8) / SEGW, j0 = cc * 8 - e * SEGW;
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const int ja = j0 + 2 * h, jb = ja + 1;
        const uint32_t lo = ja < N_OUT ? split_term(v[ja < N_OUT ? ja : 0], e) : 0;
        const uint32_t hi = jb < N_OUT ? split_term(v[jb < N_OUT ? jb : 0], e) : 0;
        w[h] = lo | (hi << 16);
      }
      MHC_ST(reinterpret_cast<uint4*>(row + cc * 128), make_uint4(w[0], w[1], w[2], w[3]));
    }
  }
}

// B1 for one token t, one warp (src/backward/golden.py:51-62, 74, 77-86, 89):
//   dh_pre[i] = sum_d dh_in[d] x[i,d]; dh_pre2, dh_post2; dh_mix = tmp * inv_rms;
//   c = (sum_j tmp_j h_mix_j) inv_rms^3 / nD
// writes rec[t] = {dh_mix[0..N), c, h_pre[0..n), 0...} and adds the token's
// dalpha (3) and dbias (N) terms to the warp's running sums.  Needs
// D % 8 == 0 and 16-byte aligned x / dh_in.
template <int n>
__device__ __forceinline__ void bwd_row_token(const BwdRowArgs& a, int64_t t, int lane, RowAcc<n>& acc) {
  using R = Rec<n>;
  constexpr int N_OUT = R::N_OUT;
  constexpr int M = RowAcc<n>::M;
  const int D = a.D;
  const int nD = n * D;
  const float a_pre = MHC_LDG(a.alpha), a_post = MHC_LDG(a.alpha + 1), a_res = MHC_LDG(a.alpha + 2);
  // small per-token inputs first, so they are in flight during the row stream
  float hm[M], gin[M], dpo[M];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const int jj = lane + 32 * m;
    hm[m] = gin[m] = dpo[m] = 0.f;
    if (jj < N_OUT) {
      hm[m] = MHC_LDG(a.h_mix + t * N_OUT + jj);
      if (jj < n) {
        gin[m] = MHC_LDG(a.h_pre + t * n + jj);
      } else if (jj < 2 * n) {
        gin[m] = MHC_LDG(a.h_post + t * n + (jj - n));
        dpo[m] = MHC_LDG(a.dh_post + t * n + (jj - n));
      } else {
        gin[m] = MHC_LDG(a.dh_res + t * (n * n) + (jj - 2 * n));
      }
    }
  }
  const float ir = MHC_LDG(a.inv_rms + t);

  const uint16_t* xr = a.x + t * nD;
  const uint16_t* gr = a.dh_in + t * D;
  float p[n];
#pragma unroll
  for (int i = 0; i < n; ++i) p[i] = 0.f;
  // 256-element chunks in flight per lane: U (n + 1) 16-byte loads, ~300
  // bytes per lane whatever n, inside the 128 registers a 512-thread CTA
  // allows (U = 4 at n = 8 alone took them all and spilled)
  constexpr int U = n <= 6 ? 4 : (n == 7 ? 3 : 2);
  for (int c0 = 0; c0 < D; c0 += 256 * U) {
    uint4 g[U], xv[U][n];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int d = c0 + u * 256 + lane * 8;
      if (d < D) {
        g[u] = ldg_stream(gr + d);
#pragma unroll
        for (int i = 0; i < n; ++i) xv[u][i] = ldg_stream(xr + i * D + d);
      } else {
        g[u] = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < n; ++i) xv[u][i] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float gf[8];
      bf16x8(g[u], gf);
#pragma unroll
      for (int i = 0; i < n; ++i) {
        float xf[8];
        bf16x8(xv[u][i], xf);
        float s0 = gf[0] * xf[0], s1 = gf[1] * xf[1];
        s0 = fmaf(gf[2], xf[2], s0);
        s1 = fmaf(gf[3], xf[3], s1);
        s0 = fmaf(gf[4], xf[4], s0);
        s1 = fmaf(gf[5], xf[5], s1);
        s0 = fmaf(gf[6], xf[6], s0);
        s1 = fmaf(gf[7], xf[7], s1);
        p[i] += s0 + s1;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < n; ++i) p[i] = warp_sum(p[i]);

  float* rt = a.rec + t * R::W;
  float dinv = 0.f, dal0 = 0.f, dal1 = 0.f, dal2 = 0.f;
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const int jj = lane + 32 * m;
    if (jj < N_OUT) {
      float g2, tmp;
      if (jj < n) {
        float dp = p[0];
#pragma unroll
        for (int i = 1; i < n; ++i)
          if (jj == i) dp = p[i];
        const float s = gin[m] - a.hc_eps;
        g2 = dp * s * (1.0f - s);                 // golden.py:54
        tmp = a_pre * g2;
      } else if (jj < 2 * n) {
        const float hq = gin[m];
        g2 = dpo[m] * hq * (1.0f - hq / 2.0f);    // golden.py:55
        tmp = a_post * g2;
      } else {
        g2 = gin[m];
        tmp = a_res * g2;
      }
      MHC_ST(rt + jj, tmp * ir);                  // dh_mix (golden.py:62)
      acc.b[m] += g2;                             // dbias terms (golden.py:83-85)
      const float dal = g2 * (hm[m] * ir);        // dalpha terms (golden.py:77-79)
      if (jj < n) dal0 += dal;
      else if (jj < 2 * n) dal1 += dal;
      else dal2 += dal;
      dinv += tmp * hm[m];
    }
  }
  dinv = warp_sum(dinv);                          // golden.py:74
  dal0 = warp_sum(dal0);
  dal1 = warp_sum(dal1);
  dal2 = warp_sum(dal2);
  if (lane == 0) {
    MHC_ST(rt + N_OUT, dinv * (ir * ir * ir) * (1.0f / (float)nD));   // c (golden.py:89)
    acc.al0 += dal0;
    acc.al1 += dal1;
    acc.al2 += dal2;
  }
  // record tail: h_pre[lane] is this lane's gin[0] (loaded before the row
  // stream), so the record needs no second load of it
  static_assert(R::W - N_OUT - 1 <= 32, "record tail wider than a warp");
  if (N_OUT + 1 + lane < R::W) MHC_ST(rt + N_OUT + 1 + lane, lane < n ? gin[0] : 0.f);
}

// B1 over all tokens: token t is owned by global warp t % W, so every sum
// has a fixed order; each warp writes its dalpha / dbias partial row to
// abpart[warp][CW].
template <int n>
__global__ void __launch_bounds__(kThreads, 1) bwd_rows_kernel(const BwdRowArgs a, float* __restrict__ abpart,
                                                                int64_t T) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int64_t W = (int64_t)gridDim.x * kWarps;
  // The split phi * gamma images first, one 64-k block per warp, from the
  // last warp down: the last warps own a token fewer when T % W != 0.
  if (a.img != nullptr)
    for (int64_t b = W - 1 - gw; b < a.img_blocks; b += W) split_image_block<n>(a, (int)b, lane);
  RowAcc<n> acc;
  for (int64_t t = gw; t < T; t += W) bwd_row_token<n>(a, t, lane, acc);
  acc.store(abpart + gw * Rec<n>::CW, lane);
}

// Forward, row half (src/forward/golden.py:34-69), per token t: sum the S_K
// partial rows [h_mix (N_OUT), sum x^2] the projection parked in h_in's row t,
// in slice order; inv_rms = 1/sqrt(sum x^2 / nD + norm_eps); gates from
// h_mix * inv_rms; then h_in[t, d] = bf16(sum_i h_pre[t,i] x[t,i,d]) streamed
// over the row (all partial loads of the warp complete, through the
// shuffles, before its first h_in store).  The partials are read with plain
// (coherent) loads: in the fused forward other CTAs wrote them during the
// same launch.  Needs D % 8 == 0 and 16-byte aligned x / h_in.
struct FwdRowArgs {
  const uint16_t* x;
  const float* alpha;   // [3]
  const float* bias;    // [N_OUT]
  uint16_t* h_in;
  float* h_post;
  float* h_res;
  float* inv_rms;   // optional
  float* h_mix;     // optional
  float* h_pre;     // optional
  float* h_in_rstd; // optional: 1/sqrt(mean(h_in^2) + h_in_eps) over the bf16 row, the next RMSNorm's factor
  const uint8_t* x8;     // optional: x as e4m3 bytes [T, n, D] (then x is unused) ...
  const int8_t* x_exp;   // ... with x = x8 * 2^x_exp[t] (NULL: exponent 0)
  int D, S_K, RW;
  float norm_eps, hc_eps, h_in_eps;
};

// Per-warp constants: alpha and this lane's bias entries.
template <int n>
struct FwdRow {
  static constexpr int N_OUT = n * n + 2 * n;
  static constexpr int M = (N_OUT + 1 + 31) / 32;   // partial columns per lane (N_OUT outputs + sum x^2)
  float a_pre, a_post, a_res, inv_nd;
  float bj[M];
  __device__ __forceinline__ void load(const FwdRowArgs& a, int lane) {
    a_pre = MHC_LDG(a.alpha);
    a_post = MHC_LDG(a.alpha + 1);
    a_res = MHC_LDG(a.alpha + 2);
    inv_nd = 1.0f / (float)(n * a.D);
#pragma unroll
    for (int m = 0; m < M; ++m) bj[m] = (lane + 32 * m) < N_OUT ? MHC_LDG(a.bias + lane + 32 * m) : 0.f;
  }
};

// Steps (1) and (2) of token t; returns h_pre[t, lane] in lanes 0..n-1.
// After it returns, every lane is done with the partials in h_in's row t.
template <int n>
__device__ __forceinline__ float fwd_row_gates(const FwdRowArgs& a, const FwdRow<n>& k, int64_t t, int lane) {
  constexpr int N_OUT = FwdRow<n>::N_OUT;
  constexpr int M = FwdRow<n>::M;
  const int D = a.D;
  // (1) partial rows of token t, summed in slice order
  const float* pr = reinterpret_cast<const float*>(a.h_in + t * D);
  float hm[M];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const int c = lane + 32 * m;
    float acc = 0.f;
    if (c <= N_OUT) {
      // kBatch loads in flight before their adds (still in slice order): the
      // partials come from L2, and one round trip per slice would dominate
      // the token's time.  Slices past S_K add an exact 0.
      constexpr int kBatch = 16;
      for (int k0 = 0; k0 < a.S_K; k0 += kBatch) {
        float v[kBatch];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) v[b] = k0 + b < a.S_K ? MHC_LD(pr + (k0 + b) * a.RW + c) : 0.f;
#pragma unroll
        for (int b = 0; b < kBatch; ++b) acc += v[b];
      }
    }
    hm[m] = acc;
  }
  const float sq = __shfl_sync(0xffffffffu, hm[N_OUT / 32], N_OUT % 32);
  const float ir = 1.0f / sqrtf(sq * k.inv_nd + a.norm_eps);
  // (2) gates and the fp32 outputs
  float hp_lane = 0.f;
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const int jj = lane + 32 * m;
    if (jj < N_OUT) {
      const float v = hm[m] * ir;
      if (jj < n) {
        hp_lane = sigmoid_acc(k.a_pre * v + k.bj[m]) + a.hc_eps;
        if (a.h_pre) MHC_ST(a.h_pre + t * n + jj, hp_lane);
      } else if (jj < 2 * n) {
        MHC_ST(a.h_post + t * n + (jj - n), 2.0f * sigmoid_acc(k.a_post * v + k.bj[m]));
      } else {
        MHC_ST(a.h_res + t * (n * n) + (jj - 2 * n), k.a_res * v + k.bj[m]);
      }
      if (a.h_mix) MHC_ST(a.h_mix + t * N_OUT + jj, hm[m]);
    }
  }
  if (lane == 0 && a.inv_rms) MHC_ST(a.inv_rms + t, ir);
  // Every lane has used its partials (the stores above consume them): only
  // now may row t of h_in, which holds them, be overwritten.
  __syncwarp();
  asm volatile("" ::: "memory");
  return hp_lane;
}

// kFp8: x comes as e4m3 bytes (a.x8, scaled by 2^a.x_exp[t]) instead of bf16.
// kU: 256-element chunks of x in flight per lane (0: the default for n).
template <int n, bool kFp8 = false, int kU = 0>
__device__ __forceinline__ void fwd_row_token(const FwdRowArgs& a, const FwdRow<n>& k, int64_t t, int lane) {
  const int D = a.D;
  const int64_t nD = (int64_t)n * D;
  const float hp_lane = fwd_row_gates<n>(a, k, t, lane);
  float hp[n];
#pragma unroll
  for (int i = 0; i < n; ++i) hp[i] = __shfl_sync(0xffffffffu, hp_lane, i);
  uint16_t* hr = a.h_in + t * D;
  float sq = 0.f;   // sum of the bf16 h_in values squared (when h_in_rstd is asked for)
  if constexpr (kFp8) {
    // (3, fp8 x) h_in = sum_i (h_pre[i] 2^e) x8[i, :]: scaling the weights by
    // the power of two instead of each x value gives the same products, so
    // the result is the one of the bf16 forward on x = x8 2^e, bit for bit
    const float sc = a.x_exp ? ldexpf(1.0f, (int)MHC_LDG(a.x_exp + t)) : 1.0f;
#pragma unroll
    for (int i = 0; i < n; ++i) hp[i] *= sc;
    const uint8_t* xr8 = a.x8 + t * nD;
    constexpr int U8 = 2;   // 512-element chunks in flight per lane (16 bytes per stream)
    for (int c0 = 0; c0 < D; c0 += 512 * U8) {
      uint4 xv[U8][n];
#pragma unroll
      for (int u = 0; u < U8; ++u) {
        const int d = c0 + u * 512 + lane * 16;
#pragma unroll
        for (int i = 0; i < n; ++i) xv[u][i] = d < D ? ldg_stream(xr8 + (int64_t)i * D + d) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < U8; ++u) {
        const int d = c0 + u * 512 + lane * 16;
        if (d < D) {
          // two halves of 8 elements (words 2hh, 2hh+1 of each stream's 16
          // bytes), so only 8 sums are live at a time
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float acc[8];
#pragma unroll
            for (int i = 0; i < n; ++i) {
              const uint32_t w[2] = {hh ? xv[u][i].z : xv[u][i].x, hh ? xv[u][i].w : xv[u][i].y};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint32_t pair = w[q / 2] >> (16 * (q & 1));
                const __half2_raw h2 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(pair & 0xFFFFu), __NV_E4M3);
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
                if (i == 0) {
                  acc[2 * q] = hp[0] * f.x;
                  acc[2 * q + 1] = hp[0] * f.y;
                } else {
                  acc[2 * q] = fmaf(hp[i], f.x, acc[2 * q]);
                  acc[2 * q + 1] = fmaf(hp[i], f.y, acc[2 * q + 1]);
                }
              }
            }
            uint4 o;
            o.x = pack_bf16x2(acc[0], acc[1]);
            o.y = pack_bf16x2(acc[2], acc[3]);
            o.z = pack_bf16x2(acc[4], acc[5]);
            o.w = pack_bf16x2(acc[6], acc[7]);
            MHC_ST(reinterpret_cast<uint4*>(hr + d + 8 * hh), o);
            if (a.h_in_rstd) {
              float r[8];
              bf16x8(o, r);
#pragma unroll
              for (int e = 0; e < 8; ++e) sq = fmaf(r[e], r[e], sq);
            }
          }
        }
      }
    }
    if (a.h_in_rstd) {
      sq = warp_sum(sq);
      if (lane == 0) MHC_ST(a.h_in_rstd + t, 1.0f / sqrtf(sq / (float)D + a.h_in_eps));
    }
  } else {
  // (3) h_in = sum_i h_pre[i] x[i, :], streamed (U 256-element chunks in flight per lane)
  const uint16_t* xr = a.x + t * nD;
  constexpr int U = kU > 0 ? kU : (n <= 4 ? 4 : 2);
  for (int c0 = 0; c0 < D; c0 += 256 * U) {
    uint4 xv[U][n];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int d = c0 + u * 256 + lane * 8;
#pragma unroll
      for (int i = 0; i < n; ++i) xv[u][i] = d < D ? ldg_stream(xr + (int64_t)i * D + d) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int d = c0 + u * 256 + lane * 8;
      if (d < D) {
        float acc[8];
        {
          float f[8];
          bf16x8(xv[u][0], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = hp[0] * f[e];
        }
#pragma unroll
        for (int i = 1; i < n; ++i) {
          float f[8];
          bf16x8(xv[u][i], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = fmaf(hp[i], f[e], acc[e]);
        }
        uint4 o;
        o.x = pack_bf16x2(acc[0], acc[1]);
        o.y = pack_bf16x2(acc[2], acc[3]);
        o.z = pack_bf16x2(acc[4], acc[5]);
        o.w = pack_bf16x2(acc[6], acc[7]);
        MHC_ST(reinterpret_cast<uint4*>(hr + d), o);
        if (a.h_in_rstd) {
          float r[8];
          bf16x8(o, r);
#pragma unroll
          for (int e = 0; e < 8; ++e) sq = fmaf(r[e], r[e], sq);
        }
      }
    }
  }
  if (a.h_in_rstd) {
    sq = warp_sum(sq);
    if (lane == 0) MHC_ST(a.h_in_rstd + t, 1.0f / sqrtf(sq / (float)D + a.h_in_eps));
  }
  }
}

// Forward, second kernel of the two-kernel forward: warp t % W takes token t.
template <int n, bool kFp8 = false>
__global__ void __launch_bounds__(kThreads, 1) fwd_rows_kernel(const FwdRowArgs a, int64_t T) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int64_t W = (int64_t)gridDim.x * kWarps;
  FwdRow<n> k;
  k.load(a, lane);
  for (int64_t t = gw; t < T; t += W) fwd_row_token<n, kFp8>(a, k, t, lane);
}

}  // namespace rowdot
}  // namespace mhc
