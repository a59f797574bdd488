// Backward for the shapes the n = 4 tensor-core backward does not take (n other
// than 4: the n = 8 "wide" hyper-connection above all): dx and the
// parameter-gradient product on the tensor cores, dx on the CUDA cores
// (dx_kernel) when D is not a multiple of 64.
//
// Math: src/backward/golden.py:38-96, split as in the tensor-core backward:
//   * rowdot::bwd_rows_kernel<n> leaves one record per token, {dh_mix[N], c,
//     h_pre[n]} (golden.py:49-62, 74, 89), and the dalpha/dbias partials;
//   * dx[t,k] = (sum_j dh_mix[t,j] phi[j,k]) gamma[k] - c[t] x[t,k]
//     + h_pre[t,i] dh_in[t,d]  (k = i*D + d; golden.py:65, 89-94):
//     - D % 64 == 0: split phi * gamma images per 64-k block (built by the
//       row kernel's warps, rowdot::split_image_block),
//       then dx_tc_pair_kernel (even n: pairs of streams over one d-range,
//       N = 128 MMAs) or dx_tc_kernel (odd n: one 64-k block at a time),
//       both with the tile's dh_mix terms in tensor memory (below);
//     - otherwise transpose_kernel (the records' dh_mix into dmT [N][Tp],
//       token fastest) and dx_kernel, a [T,N] x [N,nD] product tiled through
//       shared memory (cp.async), 64 tokens x 256 k per CTA, 8 x 8 outputs
//       per thread, the N-term sum in fp32 FMAs in ascending j;
//   * gimg_kernel + g_tc_kernel: gpart[g][j][k] = sum over the tokens of
//     token group g of dh_mix[t,j] x[t,k] (the un-scaled dphi,
//     golden.py:68-69) on the tensor cores (below);
//   * generic::finalize_param_kernel (dphi, dgamma and the dalpha / dbias
//     column sums) as in the tensor-core backward (fixed order, so results
//     repeat bit for bit).
// Needs D % 8 == 0 and 16-byte aligned x, dh_in, dx, phi and gamma.
#pragma once

#include "common.cuh"
#include "bwd_sm100.cuh"
#include "sm100.cuh"

#undef MHC_FILE_ID
#define MHC_FILE_ID 4   // debug-bounds site ids: 4 * 100000 + line

namespace mhc {
namespace tiled {

constexpr int kThreads = 256;
constexpr int kTT = 64;    // tokens per dx tile (8 warps x 8 tokens)
constexpr int kKL = 8;     // consecutive k per lane (one 16-byte bf16 load)
constexpr int kKT = 32 * kKL;   // k per tile

template <int n>
struct Dims {
  static constexpr int N = n * n + 2 * n;
  static constexpr int RW = ((N + 1 + n) + 3) / 4 * 4;   // record width (rowdot::Rec<n>::W)
  // dx_kernel's dynamic shared memory: dmT [N][kTT], ph [N][kKT], c [kTT], h_pre [kTT][n]
  static constexpr int DX_SMEM = 4 * (N * kTT + N * kKT + kTT + kTT * n);
};

// Tokens of the transposed dh_mix (a whole number of dx tiles).
inline int64_t padded_tokens(int64_t T) { return (T + kTT - 1) / kTT * kTT; }

__device__ __forceinline__ void cp16(void* dst_smem, const void* src) {
  src = MHC_LDP(src, 16);
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
    tile[r][tx] = (t < T && j < N) ? MHC_LDG(rec + t * RW + j) : 0.f;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += kThreads / 32) {
    const int j = j0 + r;
    const int64_t t = t0 + tx;
    if (j < N && t < Tp) MHC_ST(dmT + (int64_t)j * Tp + t, tile[tx][r]);
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
    const float v = t < T ? MHC_LDG(rec + t * RW + N + c) : 0.f;
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
    const float4 g0 = MHC_LDG(reinterpret_cast<const float4*>(gamma + k));
    const float4 g1 = MHC_LDG(reinterpret_cast<const float4*>(gamma + k + 4));
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
    const uint4 xr = MHC_LDG(reinterpret_cast<const uint4*>(x + t * nD + k));
    const uint4 gr = MHC_LDG(reinterpret_cast<const uint4*>(dh_in + t * D + d));
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
    MHC_ST(reinterpret_cast<uint4*>(dx + t * nD + k), make_uint4(w[0], w[1], w[2], w[3]));
  }
}

// ------------------------------------------------------------------ G on the tensor cores
// gpart[g][j][k] = sum over the tokens of token group g of (hi + mid)[t,j] x[t,k],
// with hi and mid the first two bf16 terms of dh_mix (G needs ~2^-17, as in
// the n = 4 tensor-core backward).
//   * gimg_kernel writes, once per 128-token tile, the tile's DHM image
//     [128 tok x (hi | mid)] (K-major interleaved) into the workspace;
//   * g_tc_kernel: CTA (k-range of 128, token group g) walks the tiles g,
//     g + S_T, ...  W0 loads per tile the x block [128 tok x 128 k] as two
//     128-B-swizzled TMA boxes and the tile's DHM image (bulk copy, from L2:
//     every k-range reads it) into one stage of a GS-deep ring; W1 issues 8
//     tcgen05.mma per tile (M = 128 k, x read MN-major; N = the hi and mid
//     segments, DHM read MN-major; K = 16 tokens each) into one of two TMEM
//     accumulators; WG_E (thread = k row = TMEM lane) adds each tile's
//     hi + mid into fp32 registers in tile order and stores its row of the
//     group's partial once.
// Every wait is bounded (sm100::mbar_wait): a broken pipeline ends with
// MHC_ERR_DEVICE_TIMEOUT in the status word instead of hanging.
constexpr int kGThreads = 6 * 32;   // W0, W1, WG_E(4)

template <int n>
struct GCfg {
  static constexpr int N_OUT = n * n + 2 * n;
  static constexpr int SEGW = (N_OUT + 15) / 16 * 16;   // one term segment (MMA N per term)
  static constexpr int KA = 2 * SEGW;                    // hi | mid
  static constexpr int RG = (KA / 8) * 128;              // one 8-row group of the DHM image
  static constexpr int DHM_BYTES = 16 * RG;              // 128 token rows
  static constexpr int BOX_BYTES = 128 * 128;            // one {64 k, 128 tok} x box
  static constexpr int STAGE_BYTES = 2 * BOX_BYTES + DHM_BYTES;
  static constexpr int GS = (232448 - 1024 - 256) / STAGE_BYTES < 6 ? (232448 - 1024 - 256) / STAGE_BYTES : 6;
  static constexpr int RW = Dims<n>::RW;
  static constexpr int ACC_COLS = (KA + 31) / 32 * 32;
  static constexpr int TMEM_COLS = 2 * ACC_COLS <= 32 ? 32 : 2 * ACC_COLS <= 64 ? 64 : 2 * ACC_COLS <= 128 ? 128
                                   : 2 * ACC_COLS <= 256 ? 256 : 512;
  static constexpr int SMEM = 1024 + GS * STAGE_BYTES + 256;
  static_assert(KA <= 256 && KA % 16 == 0, "UMMA N");
  static_assert(STAGE_BYTES % 1024 == 0, "stages keep the 128-B swizzle atoms aligned");
  static_assert(GS >= 2, "ring depth");
  static_assert(2 * ACC_COLS <= 512, "TMEM");
  static_assert(SMEM <= 232448, "shared memory");
};

// DHM image of tile blockIdx.x: row = token, column e * SEGW + j = bf16 term
// e (0 = hi, 1 = mid) of dh_mix[t][j] (zeros for j >= N_OUT and t >= T),
// K-major interleaved, as g_tc_kernel's B operand reads it.  128 threads,
// thread = token row.
template <int n>
__global__ void __launch_bounds__(128) gimg_kernel(const float* __restrict__ rec, uint8_t* __restrict__ img,
                                                   int64_t T) {
  using Cf = GCfg<n>;
  constexpr int N_OUT = Cf::N_OUT;
  const int row = threadIdx.x;
  const int64_t t = (int64_t)blockIdx.x * 128 + row;
  float r[Cf::SEGW];
#pragma unroll
  for (int c = 0; c < Cf::SEGW; ++c) r[c] = 0.f;
  if (t < T) {
    const float4* rp = reinterpret_cast<const float4*>(rec + t * Cf::RW);
#pragma unroll
    for (int c4 = 0; c4 < Cf::SEGW / 4; ++c4) {
      if (4 * c4 < N_OUT) {
        const float4 v = MHC_LDG(rp + c4);
        r[4 * c4] = v.x;
        r[4 * c4 + 1] = v.y;
        r[4 * c4 + 2] = v.z;
        r[4 * c4 + 3] = v.w;
      }
    }
#pragma unroll
    for (int c = N_OUT; c < Cf::SEGW; ++c) r[c] = 0.f;   // c, h_pre and padding of the record
  }
  uint8_t* dst = img + (size_t)blockIdx.x * Cf::DHM_BYTES;
#pragma unroll
  for (int kc = 0; kc < Cf::KA / 8; ++kc) {
    const int e = (kc * 8) / Cf::SEGW, j0 = kc * 8 - e * Cf::SEGW;
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const uint32_t lo = split_term(r[j0 + 2 * h], e);
      const uint32_t hi = split_term(r[j0 + 2 * h + 1], e);
      w[h] = lo | (hi << 16);
    }
    MHC_ST(reinterpret_cast<uint4*>(dst + bwdtc::interleave_off(row, kc * 8, Cf::RG)), make_uint4(w[0], w[1], w[2], w[3]));
  }
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  if (!MHC_CHK(src, bytes)) return;   // the barrier's expect_tx then runs into its bounded wait
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

template <int n>
__global__ void __launch_bounds__(kGThreads, 1)
    g_tc_kernel(const __grid_constant__ CUtensorMap map_x, const uint8_t* __restrict__ gimg, float* __restrict__ gpart,
                int* status, int nD, int S_T, int num_tiles) {
  using namespace sm100;
  using Cf = GCfg<n>;
  constexpr int N_OUT = Cf::N_OUT;
  constexpr int GS = Cf::GS;
  // barrier slots
  constexpr int FULL = 0, EMPTY = GS, ACC_FULL = 2 * GS, ACC_EMPTY = 2 * GS + 2, NBARS = 2 * GS + 4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(stages + GS * Cf::STAGE_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int k0 = blockIdx.x * 128;
  const int group = blockIdx.y;
  const int my_tiles = group < num_tiles ? (num_tiles - 1 - group) / S_T + 1 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < GS; ++i) {
      mbar_init(bar(FULL + i), 1);
      mbar_init(bar(EMPTY + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(ACC_FULL + i), 1);
      mbar_init(bar(ACC_EMPTY + i), 4);
    }
    *abort_flag = 0;
    fence_mbarrier_init_cluster();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cf::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) prefetch_tensormap(&map_x);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtx wc{abort_flag, status};

  if (warp == 0) {
    // ---------------------------------------------------------- W0: x block and DHM image per tile
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      for (int j = 0; j < my_tiles; ++j) {
        const int s = j % GS;
        const int tile = group + j * S_T;
        mbar_wait(bar(EMPTY + s), ((j / GS) & 1) ^ 1, wc);
        if (*abort_flag) continue;
        const uint32_t dst = smem_u32(stages + s * Cf::STAGE_BYTES);
        mbar_arrive_expect_tx(bar(FULL + s), Cf::STAGE_BYTES);
        tma_load_2d(dst, &map_x, bar(FULL + s), k0, tile * 128, pol);
        tma_load_2d(dst + Cf::BOX_BYTES, &map_x, bar(FULL + s), k0 + 64, tile * 128, pol);
        bulk_g2s(dst + 2 * Cf::BOX_BYTES, gimg + (size_t)tile * Cf::DHM_BYTES, Cf::DHM_BYTES, bar(FULL + s));
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- W1: MMA
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, Cf::KA, true, true);
      for (int j = 0; j < my_tiles; ++j) {
        const int s = j % GS, hb = j & 1;
        mbar_wait(bar(FULL + s), (j / GS) & 1, wc);
        mbar_wait(bar(ACC_EMPTY + hb), ((j >> 1) & 1) ^ 1, wc);
        tc_fence_after();
        if (*abort_flag) continue;
        const uint32_t st = smem_u32(stages + s * Cf::STAGE_BYTES);
        const uint64_t a = desc_mnmajor_sw128(st, Cf::BOX_BYTES, 1024);
        const uint64_t b = bwdtc::desc_kmajor_interleave(st + 2 * Cf::BOX_BYTES, Cf::RG, 128);
        const uint32_t d = tmem_base + hb * Cf::ACC_COLS;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_bf16(d, a + ((ks * 2048) >> 4), b + ((ks * 2 * Cf::RG) >> 4), idesc, ks != 0);
        umma_commit(bar(EMPTY + s));
        umma_commit(bar(ACC_FULL + hb));
      }
    }
  } else {
    // ---------------------------------------------------------- WG_E: fold, store
    const int q4 = warp & 3;
    const int row = 32 * q4 + lane;   // k row of the accumulator (TMEM lane)
    float acc[N_OUT];
#pragma unroll
    for (int c = 0; c < N_OUT; ++c) acc[c] = 0.f;
    for (int j = 0; j < my_tiles; ++j) {
      const int hb = j & 1;
      mbar_wait(bar(ACC_FULL + hb), (j >> 1) & 1, wc);
      tc_fence_after();
      const uint32_t ta = tmem_base + hb * Cf::ACC_COLS + ((uint32_t)(32 * q4) << 16);
#pragma unroll
      for (int c16 = 0; c16 < Cf::SEGW / 16; ++c16) {
        float hi[16], mid[16];
        tmem_ld16(ta + c16 * 16, hi);
        tmem_ld16(ta + Cf::SEGW + c16 * 16, mid);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int jj = c16 * 16 + e;
          if (jj < N_OUT) acc[jj] += mid[e] + hi[e];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(ACC_EMPTY + hb));
    }
    const int k = k0 + row;
    if (k < nD && !*abort_flag) {
      float* gp = gpart + (int64_t)group * N_OUT * nD + k;
#pragma unroll
      for (int jj = 0; jj < N_OUT; ++jj) MHC_ST(gp + (int64_t)jj * nD, acc[jj]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cf::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ dx on the tensor cores
// dvecX = dh_mix @ (phi * gamma) as in the n = 4 tensor-core backward: dh_mix
// and phi * gamma each split into three bf16 terms (hi, mid, lo), six term
// products summed smallest first (m.M, l.H, h.L, m.H, h.M, h.H; exact to
// ~2^-23), then dx = dvecX - c x + h_pre[i] dh_in in fp32 and rounded once.
// CTA = (128-token tile, range of 64-k blocks taken in stream-fastest order,
// so the n blocks that read one dh_in box run back to back and the box is
// read from DRAM once):
//   * WG_E (4 warps, thread = token row) writes the tile's DHM [128 tok x 3
//     segments] once into tensor memory (lane = token row, two bf16 per
//     column): the A operand of every block's products, read by the tensor
//     core without shared-memory traffic;
//   * W0 streams per 64-k block the x and dh_in boxes (TMA, 128-B swizzle)
//     and the block's split phi * gamma image (bulk copy from the image
//     row kernel leaves in the workspace) into an ST-deep ring;
//   * W1 issues 6 x SEGW/16 tcgen05.mma (M = 128 tokens, N = 64 k, K = 16,
//     A from tensor memory) per block into one of two TMEM accumulators;
//   * WG_E reads the accumulator (TMEM lane = token row), adds -c x + h_pre
//     dh_in, writes the 64 dx values of its row into a 128-B-swizzled
//     staging box (two, alternating) and one thread stores the box with TMA
//     (rows past T are clipped by the tensor map).
template <int n>
struct DxCfg {
  static constexpr int N_OUT = n * n + 2 * n;
  static constexpr int SEGW = (N_OUT + 15) / 16 * 16;
  static constexpr int KA = 3 * SEGW;                    // hi | mid | lo
  static constexpr int RG = (KA / 8) * 128;              // one 8-row group of a K-major interleaved image
  static constexpr int PH_BYTES = 8 * RG;                // 64 k rows: split phi * gamma of one 64-k block
  static constexpr int BOX_BYTES = 128 * 128;            // one {64, 128} bf16 box
  static constexpr int STAGE_BYTES = 2 * BOX_BYTES + PH_BYTES;   // x, dh_in, phi image
  static constexpr int OUT_BUFS = 2;                     // dx staging boxes
  static constexpr int ST_FIT = (232448 - 1024 - 256 - OUT_BUFS * BOX_BYTES) / STAGE_BYTES;
  static constexpr int ST = ST_FIT < 4 ? ST_FIT : 4;
  static constexpr int DHM_COL = 128;                    // TMEM: accumulators 0..127, DHM from here
  static constexpr int TMEM_COLS = 256;
  static constexpr int RW = Dims<n>::RW;
  static constexpr int SMEM = 1024 + ST * STAGE_BYTES + OUT_BUFS * BOX_BYTES + 256;
  static_assert(STAGE_BYTES % 1024 == 0, "stages keep the 128-B swizzle atoms aligned");
  static_assert(ST >= 2, "ring depth");
  static_assert(DHM_COL + KA / 2 <= TMEM_COLS, "TMEM");
  static_assert(SMEM <= 232448, "shared memory");
};

template <int n>
__global__ void __launch_bounds__(kGThreads, 1)
    dx_tc_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_dh,
                 const __grid_constant__ CUtensorMap map_dx, const uint8_t* __restrict__ img,
                 const float* __restrict__ rec, int* status, int64_t T, int D, int kb_per) {
  using namespace sm100;
  using Cf = DxCfg<n>;
  constexpr int N_OUT = Cf::N_OUT;
  constexpr int ST = Cf::ST;
  constexpr int FULL = 0, EMPTY = ST, ACC_FULL = 2 * ST, ACC_EMPTY = 2 * ST + 2, DHM_FULL = 2 * ST + 4,
                NBARS = 2 * ST + 5;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* outb = stages + ST * Cf::STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(outb + Cf::OUT_BUFS * Cf::BOX_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int nD = n * D;
  const int KB = nD / 64;
  const int tile = blockIdx.x;
  const int kb0 = blockIdx.y * kb_per;
  const int nkb = max(0, min(kb_per, KB - kb0));
  // the CTA's blocks in stream-fastest order: position q -> block (q % n) *
  // D/64 + q / n, so the n blocks that share one dh_in box follow each other
  const int DB = D / 64;
  auto kb_of = [&](int q) { return (q % n) * DB + q / n; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(bar(FULL + i), 1);
      mbar_init(bar(EMPTY + i), 1 + 4);   // MMA commit + the 4 epilogue warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(ACC_FULL + i), 1);
      mbar_init(bar(ACC_EMPTY + i), 4);
    }
    mbar_init(bar(DHM_FULL), 128);
    *abort_flag = 0;
    fence_mbarrier_init_cluster();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cf::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&map_x);
    prefetch_tensormap(&map_dh);
    prefetch_tensormap(&map_dx);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtx wc{abort_flag, status};

  if (warp == 0) {
    // ---------------------------------------------------------- W0: x, dh_in, phi image
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      const uint64_t pol_dh = l2_policy_evict_last();   // read again by the next n - 1 blocks
      for (int b = 0; b < nkb; ++b) {
        const int s = b % ST;
        const int kb = kb_of(kb0 + b);
        mbar_wait(bar(EMPTY + s), ((b / ST) & 1) ^ 1, wc);
        if (*abort_flag) continue;
        uint8_t* st = stages + s * Cf::STAGE_BYTES;
        mbar_arrive_expect_tx(bar(FULL + s), Cf::STAGE_BYTES);
        tma_load_2d(smem_u32(st), &map_x, bar(FULL + s), kb * 64, tile * 128, pol);
        tma_load_2d(smem_u32(st + Cf::BOX_BYTES), &map_dh, bar(FULL + s), (kb * 64) % D, tile * 128, pol_dh);
        bulk_g2s(smem_u32(st + 2 * Cf::BOX_BYTES), img + (size_t)kb * Cf::PH_BYTES, Cf::PH_BYTES, bar(FULL + s));
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- W1: MMA
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, 64, false, false);
      mbar_wait(bar(DHM_FULL), 0, wc);
      tc_fence_after();
      const uint32_t a_t = tmem_base + Cf::DHM_COL;
      for (int b = 0; b < nkb; ++b) {
        const int s = b % ST, ab = b & 1;
        mbar_wait(bar(FULL + s), (b / ST) & 1, wc);
        mbar_wait(bar(ACC_EMPTY + ab), ((b >> 1) & 1) ^ 1, wc);
        tc_fence_after();
        if (*abort_flag) continue;
        const uint64_t b_dv =
            bwdtc::desc_kmajor_interleave(smem_u32(stages + s * Cf::STAGE_BYTES + 2 * Cf::BOX_BYTES), 128, Cf::RG);
        const uint32_t d = tmem_base + ab * 64;
#pragma unroll
        for (int pr = 0; pr < 6; ++pr) {
#pragma unroll
          for (int ks = 0; ks < Cf::SEGW / 16; ++ks) {
            const uint32_t ca = (bwdtc::prod_a_term(pr) * Cf::SEGW + ks * 16) / 2;    // TMEM column
            const uint32_t cb = (bwdtc::prod_b_term(pr) * Cf::SEGW + ks * 16) * 16;   // image bytes
            umma_bf16_ta(d, a_t + ca, b_dv + (cb >> 4), idesc, pr != 0 || ks != 0);
          }
        }
        umma_commit(bar(EMPTY + s));
        umma_commit(bar(ACC_FULL + ab));
      }
    }
  } else {
    // ---------------------------------------------------------- WG_E: DHM once, dx per block
    const int q4 = warp & 3;
    const int row = 32 * q4 + lane;   // token row = TMEM lane
    const bool issuer = threadIdx.x == 64;
    const uint32_t lane_off = (uint32_t)(32 * q4) << 16;
    const int64_t t = (int64_t)tile * 128 + row;
    float c_t = 0.f, hp[n];
#pragma unroll
    for (int i = 0; i < n; ++i) hp[i] = 0.f;
    {
      float r[Cf::SEGW];
#pragma unroll
      for (int c = 0; c < Cf::SEGW; ++c) r[c] = 0.f;
      if (t < T) {
        const float* rp = rec + t * Cf::RW;
#pragma unroll
        for (int c = 0; c < N_OUT; ++c) r[c] = MHC_LDG(rp + c);
        c_t = MHC_LDG(rp + N_OUT);
#pragma unroll
        for (int i = 0; i < n; ++i) hp[i] = MHC_LDG(rp + N_OUT + 1 + i);
      }
      // term e of dh_mix[j] at TMEM column DHM_COL + (e SEGW + j) / 2 (j even: low half)
#pragma unroll
      for (int e = 0; e < 3; ++e) {
#pragma unroll
        for (int c = 0; c < Cf::SEGW / 16; ++c) {
          uint32_t w[8];
#pragma unroll
          for (int h = 0; h < 8; ++h) {
            const uint32_t lo = split_term(r[16 * c + 2 * h], e);
            const uint32_t hi = split_term(r[16 * c + 2 * h + 1], e);
            w[h] = lo | (hi << 16);
          }
          tmem_st8(tmem_base + lane_off + Cf::DHM_COL + e * (Cf::SEGW / 2) + 8 * c, w);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(DHM_FULL));
    }
    const uint64_t pol_out = l2_policy_evict_first();
    for (int b = 0; b < nkb; ++b) {
      const int s = b % ST, ab = b & 1;
      const int k0 = kb_of(kb0 + b) * 64;
      const int i = k0 / D;
      float hpi = hp[0];
#pragma unroll
      for (int ii = 1; ii < n; ++ii)
        if (i == ii) hpi = hp[ii];
      mbar_wait(bar(ACC_FULL + ab), (b >> 1) & 1, wc);
      mbar_wait(bar(FULL + s), (b / ST) & 1, wc);   // x and dh_in of the block (already complete)
      tc_fence_after();
      const uint8_t* st = stages + s * Cf::STAGE_BYTES;
      const uint32_t x_row = smem_u32(st) + row * 128;
      const uint32_t g_row = smem_u32(st + Cf::BOX_BYTES) + row * 128;
      const uint32_t o_buf = smem_u32(outb + ab * Cf::BOX_BYTES);
      const uint32_t o_row = o_buf + row * 128;
      // staging box ab is free once the store issued two blocks ago has read it
      if (issuer) bwdtc::bulk_wait_read1();
      named_sync(1, 128);
      const uint32_t ta = tmem_base + ab * 64 + lane_off;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float v0[16], v1[16];
        tmem_ld16(ta + hf * 32, v0);
        tmem_ld16(ta + hf * 32 + 16, v1);
        tmem_wait_ld();
#pragma unroll
        for (int hc = 0; hc < 4; ++hc) {
          const int c = hf * 4 + hc;   // 16-byte chunk of the 128-byte row
          const uint32_t sw = (uint32_t)((c ^ (row & 7)) << 4);
          float xf[8], gf[8];
          bwdtc::bf16x8_to_f32(bwdtc::lds128(x_row + sw), xf);
          bwdtc::bf16x8_to_f32(bwdtc::lds128(g_row + sw), gf);
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const float a0 = (hc < 2 ? v0[(hc * 8 + e) & 15] : v1[(hc * 8 + e) & 15]);
            const float a1 = (hc < 2 ? v0[(hc * 8 + e + 1) & 15] : v1[(hc * 8 + e + 1) & 15]);
            // dx = (dvecX + h_pre dh_in) - c x, two elements per packed FMA
            float2 d = __ffma2_rn(make_float2(hpi, hpi), make_float2(gf[e], gf[e + 1]), make_float2(a0, a1));
            d = __ffma2_rn(make_float2(-c_t, -c_t), make_float2(xf[e], xf[e + 1]), d);
            o[e / 2] = pack_bf16x2(d.x, d.y);
          }
          bwdtc::sts128(o_row + sw, make_uint4(o[0], o[1], o[2], o[3]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(bar(ACC_EMPTY + ab));
        mbar_arrive(bar(EMPTY + s));
      }
      fence_proxy_async_smem();
      named_sync(1, 128);
      if (issuer && !*abort_flag) {
        bwdtc::tma_store_2d(&map_dx, o_buf, k0, tile * 128, pol_out);
        bwdtc::bulk_commit();
      }
    }
    if (issuer) bwdtc::bulk_wait_all0();   // the dx stores have completed
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cf::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ dx on the tensor cores, stream pairs
// For even n: the same products as dx_tc_kernel, but a unit of work is a pair
// of 64-k blocks of streams i and i + 1 over the same d-range (consecutive in
// the stream-fastest order), so both share one dh_in box and their two split
// phi * gamma images stack into one 128-row B operand: 6 x SEGW/16
// tcgen05.mma of N = 128 per pair, half the issues of two N = 64 chains (an
// MMA costs about the same to issue at N = 64 and N = 128).  A stage holds the
// pair's two x boxes, its dh_in box and its two images; the epilogue (two
// groups of four warps, group h on block h of the pair) writes dx over the x
// boxes it has read (each thread its own row), and one thread TMA-stores them
// and releases the stage once the stores have read it.
// Two rings: XST slots of {x pair, dh_in} (read by the epilogue, dx written
// over the x boxes and stored from there) and PST slots of the pair's two
// split phi images (read by the MMA only, so released at its commit).
template <int n>
struct DxPairCfg {
  static constexpr int N_OUT = n * n + 2 * n;
  static constexpr int SEGW = (N_OUT + 15) / 16 * 16;
  static constexpr int KA = 3 * SEGW;
  static constexpr int RG = (KA / 8) * 128;
  static constexpr int PH_BYTES = 8 * RG;                // one 64-k block's image
  static constexpr int BOX_BYTES = 128 * 128;
  static constexpr int XD_BYTES = 3 * BOX_BYTES;         // x0, x1, dh_in
  static constexpr int PH2_BYTES = 2 * PH_BYTES;         // image0 | image1
  static constexpr int kBudget = 232448 - 1024 - 256;
  // as many x / dh_in slots as fit beside two image slots (at most 4), else one image slot
  static constexpr int PST = (kBudget - 2 * PH2_BYTES) / XD_BYTES >= 2 ? 2 : 1;
  static constexpr int XST_FIT = (kBudget - PST * PH2_BYTES) / XD_BYTES;
  static constexpr int XST = XST_FIT < 4 ? XST_FIT : 4;
  static constexpr int DHM_COL = 256;                    // TMEM: accumulators 0..255, DHM from here
  static constexpr int TMEM_COLS = 512;
  static constexpr int RW = Dims<n>::RW;
  static constexpr int SMEM = 1024 + XST * XD_BYTES + PST * PH2_BYTES + 256;
  static_assert(n % 2 == 0, "pairs of streams");
  static_assert(XD_BYTES % 1024 == 0 && PH2_BYTES % 1024 == 0, "slots keep the 128-B swizzle atoms aligned");
  static_assert(XST >= 2 && PST >= 1, "ring depth");
  static_assert(DHM_COL + KA / 2 <= TMEM_COLS, "TMEM");
  static_assert(SMEM <= 232448, "shared memory");
};

constexpr int kPThreads = 11 * 32;   // W0 (x, dh_in), W1 (MMA), WG_E(8), W10 (phi images)

// grid = (tiles, slices); CTA (tile, y) takes the pairs [y * kp_per, ...) of
// the nD / 128 pairs; pair p = blocks q = 2p, 2p + 1 of the stream-fastest
// order (block (q % n) * D/64 + q / n).
template <int n>
__global__ void __launch_bounds__(kPThreads, 1)
    dx_tc_pair_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_dh,
                      const __grid_constant__ CUtensorMap map_dx, const uint8_t* __restrict__ img,
                      const float* __restrict__ rec, int* status, int64_t T, int D, int kp_per) {
  using namespace sm100;
  using Cf = DxPairCfg<n>;
  constexpr int N_OUT = Cf::N_OUT;
  constexpr int XST = Cf::XST, PST = Cf::PST;
  constexpr int FULL = 0, EMPTY = XST, PFULL = 2 * XST, PEMPTY = PFULL + PST, ACC_FULL = PEMPTY + PST,
                ACC_EMPTY = ACC_FULL + 2, DHM_FULL = ACC_EMPTY + 2, NBARS = DHM_FULL + 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* images = stages + XST * Cf::XD_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(images + PST * Cf::PH2_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  const int nD = n * D;
  const int KP = nD / 128;
  const int tile = blockIdx.x;
  const int p0 = blockIdx.y * kp_per;
  const int npairs = max(0, min(kp_per, KP - p0));
  const int DB = D / 64;
  auto kb_of = [&](int q) { return (q % n) * DB + q / n; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < XST; ++i) {
      mbar_init(bar(FULL + i), 1);
      mbar_init(bar(EMPTY + i), 1);   // the store issuer once its stores have read the slot
    }
    for (int i = 0; i < PST; ++i) {
      mbar_init(bar(PFULL + i), 1);
      mbar_init(bar(PEMPTY + i), 1);  // the MMA commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(ACC_FULL + i), 1);
      mbar_init(bar(ACC_EMPTY + i), 8);   // the 8 epilogue warps
    }
    mbar_init(bar(DHM_FULL), 256);
    *abort_flag = 0;
    fence_mbarrier_init_cluster();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cf::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&map_x);
    prefetch_tensormap(&map_dh);
    prefetch_tensormap(&map_dx);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtx wc{abort_flag, status};

  if (warp == 0) {
    // ---------------------------------------------------------- W0: x pair, dh_in
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      for (int b = 0; b < npairs; ++b) {
        const int s = b % XST;
        const int q = 2 * (p0 + b);
        const int kb0 = kb_of(q), kb1 = kb_of(q + 1);
        mbar_wait(bar(EMPTY + s), ((b / XST) & 1) ^ 1, wc);
        if (*abort_flag) continue;
        const uint32_t st = smem_u32(stages + s * Cf::XD_BYTES);
        mbar_arrive_expect_tx(bar(FULL + s), Cf::XD_BYTES);
        tma_load_2d(st, &map_x, bar(FULL + s), kb0 * 64, tile * 128, pol);
        tma_load_2d(st + Cf::BOX_BYTES, &map_x, bar(FULL + s), kb1 * 64, tile * 128, pol);
        tma_load_2d(st + 2 * Cf::BOX_BYTES, &map_dh, bar(FULL + s), (kb0 * 64) % D, tile * 128, pol);
      }
    }
  } else if (warp == 10) {
    // ---------------------------------------------------------- W10: phi image pair
    if (lane == 0) {
      for (int b = 0; b < npairs; ++b) {
        const int s = b % PST;
        const int q = 2 * (p0 + b);
        const int kb0 = kb_of(q), kb1 = kb_of(q + 1);
        mbar_wait(bar(PEMPTY + s), ((b / PST) & 1) ^ 1, wc);
        if (*abort_flag) continue;
        const uint32_t im = smem_u32(images + s * Cf::PH2_BYTES);
        mbar_arrive_expect_tx(bar(PFULL + s), Cf::PH2_BYTES);
        bulk_g2s(im, img + (size_t)kb0 * Cf::PH_BYTES, Cf::PH_BYTES, bar(PFULL + s));
        bulk_g2s(im + Cf::PH_BYTES, img + (size_t)kb1 * Cf::PH_BYTES, Cf::PH_BYTES, bar(PFULL + s));
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- W1: MMA
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, 128, false, false);
      mbar_wait(bar(DHM_FULL), 0, wc);
      tc_fence_after();
      const uint32_t a_t = tmem_base + Cf::DHM_COL;
      for (int b = 0; b < npairs; ++b) {
        const int s = b % PST, ab = b & 1;
        mbar_wait(bar(PFULL + s), (b / PST) & 1, wc);
        mbar_wait(bar(ACC_EMPTY + ab), ((b >> 1) & 1) ^ 1, wc);
        tc_fence_after();
        if (*abort_flag) continue;
        // the two images stack into one 128-row K-major interleaved operand
        const uint64_t b_dv = bwdtc::desc_kmajor_interleave(smem_u32(images + s * Cf::PH2_BYTES), 128, Cf::RG);
        const uint32_t d = tmem_base + ab * 128;
#pragma unroll
        for (int pr = 0; pr < 6; ++pr) {
#pragma unroll
          for (int ks = 0; ks < Cf::SEGW / 16; ++ks) {
            const uint32_t ca = (bwdtc::prod_a_term(pr) * Cf::SEGW + ks * 16) / 2;    // TMEM column
            const uint32_t cb = (bwdtc::prod_b_term(pr) * Cf::SEGW + ks * 16) * 16;   // image bytes
            umma_bf16_ta(d, a_t + ca, b_dv + (cb >> 4), idesc, pr != 0 || ks != 0);
          }
        }
        umma_commit(bar(PEMPTY + s));
        umma_commit(bar(ACC_FULL + ab));
      }
    }
  } else {
    // ---------------------------------------------------------- WG_E: DHM once, dx per pair
    // two groups of four warps (one per TMEM lane quadrant each); group h
    // takes block h of every pair, so two warps per scheduler hide each
    // other's TMEM / shared-memory latency
    const int q4 = warp & 3;
    const int grp = (warp - 2) >> 2;
    const int row = 32 * q4 + lane;   // token row = TMEM lane
    const bool issuer = threadIdx.x == 64;
    const uint32_t lane_off = (uint32_t)(32 * q4) << 16;
    const int64_t t = (int64_t)tile * 128 + row;
    float c_t = 0.f, hp[n];
#pragma unroll
    for (int i = 0; i < n; ++i) hp[i] = 0.f;
    {
      float r[Cf::SEGW];
#pragma unroll
      for (int c = 0; c < Cf::SEGW; ++c) r[c] = 0.f;
      if (t < T) {
        const float* rp = rec + t * Cf::RW;
#pragma unroll
        for (int c = 0; c < N_OUT; ++c) r[c] = MHC_LDG(rp + c);
        c_t = MHC_LDG(rp + N_OUT);
#pragma unroll
        for (int i = 0; i < n; ++i) hp[i] = MHC_LDG(rp + N_OUT + 1 + i);
      }
      // term e of dh_mix[j] at TMEM column DHM_COL + (e SEGW + j) / 2 (j even: low half)
      // group 0 writes terms 0 and 2, group 1 term 1
#pragma unroll
      for (int e = 0; e < 3; ++e) {
        if ((e & 1) != grp) continue;
#pragma unroll
        for (int c = 0; c < Cf::SEGW / 16; ++c) {
          uint32_t w[8];
#pragma unroll
          for (int h = 0; h < 8; ++h) {
            const uint32_t lo = split_term(r[16 * c + 2 * h], e);
            const uint32_t hi = split_term(r[16 * c + 2 * h + 1], e);
            w[h] = lo | (hi << 16);
          }
          tmem_st8(tmem_base + lane_off + Cf::DHM_COL + e * (Cf::SEGW / 2) + 8 * c, w);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(DHM_FULL));
    }
    const uint64_t pol_out = l2_policy_evict_first();
    for (int b = 0; b < npairs; ++b) {
      const int s = b % XST, ab = b & 1;
      const int q = 2 * (p0 + b);
      mbar_wait(bar(ACC_FULL + ab), (b >> 1) & 1, wc);
      mbar_wait(bar(FULL + s), (b / XST) & 1, wc);   // the slot's x and dh_in boxes
      tc_fence_after();
      const uint32_t st = smem_u32(stages + s * Cf::XD_BYTES);
      const uint32_t g_row = st + 2 * Cf::BOX_BYTES + row * 128;
      {
        const int h = grp;
        const int i = (q + h) % n;   // stream of block h
        float hpi = hp[0];
#pragma unroll
        for (int ii = 1; ii < n; ++ii)
          if (i == ii) hpi = hp[ii];
        const uint32_t x_row = st + h * Cf::BOX_BYTES + row * 128;   // dx overwrites it in place
        const uint32_t ta = tmem_base + ab * 128 + h * 64 + lane_off;
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          float v0[16], v1[16];
          tmem_ld16(ta + hf * 32, v0);
          tmem_ld16(ta + hf * 32 + 16, v1);
          tmem_wait_ld();
#pragma unroll
          for (int hc = 0; hc < 4; ++hc) {
            const int c = hf * 4 + hc;   // 16-byte chunk of the 128-byte row
            const uint32_t sw = (uint32_t)((c ^ (row & 7)) << 4);
            float xf[8], gf[8];
            bwdtc::bf16x8_to_f32(bwdtc::lds128(x_row + sw), xf);
            bwdtc::bf16x8_to_f32(bwdtc::lds128(g_row + sw), gf);
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              const float a0 = (hc < 2 ? v0[(hc * 8 + e) & 15] : v1[(hc * 8 + e) & 15]);
              const float a1 = (hc < 2 ? v0[(hc * 8 + e + 1) & 15] : v1[(hc * 8 + e + 1) & 15]);
              // dx = (dvecX + h_pre dh_in) - c x, two elements per packed FMA
              float2 d = __ffma2_rn(make_float2(hpi, hpi), make_float2(gf[e], gf[e + 1]), make_float2(a0, a1));
              d = __ffma2_rn(make_float2(-c_t, -c_t), make_float2(xf[e], xf[e + 1]), d);
              o[e / 2] = pack_bf16x2(d.x, d.y);
            }
            bwdtc::sts128(x_row + sw, make_uint4(o[0], o[1], o[2], o[3]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(ACC_EMPTY + ab));
      fence_proxy_async_smem();
      named_sync(1, 256);
      if (issuer) {
        if (!*abort_flag) {
          bwdtc::tma_store_2d(&map_dx, st, kb_of(q) * 64, tile * 128, pol_out);
          bwdtc::tma_store_2d(&map_dx, st + Cf::BOX_BYTES, kb_of(q + 1) * 64, tile * 128, pol_out);
          bwdtc::bulk_commit();
          bwdtc::bulk_wait_read0();   // the stores have read the stage
        }
        mbar_arrive(bar(EMPTY + s));
      }
    }
    if (issuer) bwdtc::bulk_wait_all0();   // the dx stores have completed
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cf::TMEM_COLS);
  }
}

}  // namespace tiled
}  // namespace mhc
