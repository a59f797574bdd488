// Forward of the mHC pre-op on sm_100a: tcgen05 projection + cluster K-split.
//
// Math: src/forward/golden.py:34-69 (h_mix = x @ phi^T pre-RMS, inv_rms,
// gates, h_in = sum_i h_pre[i] * x[i,:]).
//
// Work decomposition.  Tokens are processed in tiles of 128 (the UMMA M).  A
// cluster of C CTAs owns one tile at a time; CTA r of the cluster owns the
// d-slice [r*Dc, (r+1)*Dc) of every stream, i.e. the K-subset
// {i*D + d : d in slice} of each 128-token row block.  Per tile and CTA:
//   * W0 streams x (128 x 64 bf16, 128-B swizzle) and the bf16-split phi
//     block (NB x 64) of each K-block into an S-stage ring with TMA;
//   * W1 issues tcgen05.mma (M=128 tokens, N=NB split-phi rows, K=16); every
//     K-block of 64 starts a fresh accumulator in a ring of NBUF TMEM buffers;
//   * WG_SR (4 warps, one thread per token row = TMEM lane) sums x^2 of its
//     row from the smem stage (tree sum per stage) and folds each K-block's
//     accumulator and the phi split terms into its fp32 partial h_mix with
//     round-to-nearest adds -- the tensor core's own accumulation across many
//     K steps drifts (about 2^-23 per step, one-signed), per K-block it does
//     not -- then sends (h_mix, sum x^2) of its token to the token's owner CTA
//     through DSMEM;
//   * WG_A (4 warps): the owner reduces the C partials of its tokens in fixed
//     rank order, writes h_mix / inv_rms / h_pre / h_post / h_res and
//     broadcasts h_pre to every CTA of the cluster;
//   * WG_B (4 warps) re-reads its d-slice of the tile from L2 (W2 issues 3-D
//     TMA loads, evict-first) and writes h_in for the slice.
// phi is split into NT bf16 terms (hi, mid[, lo]) stacked as UMMA N rows, so
// x (exact in bf16) times phi is exact to ~2^-(8*NT) before fp32 accumulation.
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"
#include "sm100.cuh"

#ifndef MHC_FWD_PREFETCH
#define MHC_FWD_PREFETCH 0
#endif

namespace mhc {
namespace fwdtc {

using namespace sm100;

constexpr int kBM = 128;          // tokens per tile = UMMA M = TMEM lanes
constexpr int kBK = 64;           // bf16 elements per 128-byte row
constexpr int kThreads = 15 * 32; // W0, W1, W2, WG_SR(4), WG_A(4), WG_B(4)
constexpr int kSmemLimit = 232448;

constexpr int round_up(int v, int a) { return (v + a - 1) / a * a; }
constexpr int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p *= 2;
  return p;
}

template <int n>
struct Cfg {
  static constexpr int N_OUT = n * n + 2 * n;
  static constexpr int NT = (n <= 5) ? 3 : 2;              // phi split terms
  static constexpr int NB = round_up(NT * N_OUT, 16);      // UMMA N
  static constexpr int A_BYTES = kBM * 128;
  static constexpr int B_BYTES = NB * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int RR_TOK = (n <= 4) ? 32 : 16;       // tokens per re-read stage
  static constexpr int RR_BYTES = RR_TOK * n * 128;
  static constexpr int RS = round_up(N_OUT + 1, 4);        // floats per partial row
  static constexpr int ACC_COLS = round_up(NB, 32);
  static constexpr int NBUF = (512 / ACC_COLS) < 4 ? (512 / ACC_COLS) : 4;   // accumulator ring
  static constexpr int TMEM_COLS = pow2_at_least(NBUF * ACC_COLS);
  static constexpr int R = 3;                              // re-read stages

  static constexpr int smem_bytes(int S, int RB) {
    return 1024 /*align slack*/ + S * STAGE_BYTES + R * RR_BYTES + RB * kBM * RS * 4 /*red*/ +
           RB * kBM * n * 4 /*hpre*/ + kBM * RS * 4 /*tot (owner)*/ + kBM * n * 4 /*hp_s*/ +
           512 /*barriers + slots*/;
  }
  static constexpr int RB = smem_bytes(3, 2) <= kSmemLimit ? 2 : 1;
  static constexpr int pick_stages() {
    int s = 8;
    while (s > 2 && smem_bytes(s, RB) > kSmemLimit) --s;
    return s;
  }
  static constexpr int S = pick_stages();
  static constexpr int SMEM = smem_bytes(S, RB);
  static_assert(SMEM <= kSmemLimit, "forward tile does not fit in shared memory");
  static_assert(NB <= 256, "UMMA N above 256");
  static_assert(NBUF >= 2 && TMEM_COLS <= 512, "TMEM accumulator ring");
};

struct Params {
  const float* alpha;
  const float* bias;
  uint16_t* h_in;
  float* h_post;
  float* h_res;
  float* inv_rms;
  float* h_mix;
  float* h_pre;
  int* status;
  int64_t T;
  int D;
  int Dc;       // d-slice per CTA (multiple of 64)
  int C;        // cluster size
  int num_tiles;
  float norm_eps;
  float hc_eps;
};

// Barrier slots (8 bytes each) in the barrier area.
template <int n>
struct Bars {
  using Cf = Cfg<n>;
  static constexpr int full = 0;
  static constexpr int empty = full + Cf::S;
  static constexpr int acc_full = empty + Cf::S;
  static constexpr int acc_empty = acc_full + Cf::NBUF;
  static constexpr int red_full = acc_empty + Cf::NBUF;
  static constexpr int red_free = red_full + Cf::RB;
  static constexpr int hpre_full = red_free + Cf::RB;
  static constexpr int hpre_free = hpre_full + Cf::RB;
  static constexpr int rr_full = hpre_free + Cf::RB;
  static constexpr int rr_empty = rr_full + Cf::R;
  static constexpr int count = rr_empty + Cf::R;
};

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

template <int n>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap map_x2d, const __grid_constant__ CUtensorMap map_phi,
               const __grid_constant__ CUtensorMap map_x3d, const Params p) {
  using Cf = Cfg<n>;
  using B = Bars<n>;
  constexpr int N_OUT = Cf::N_OUT;
  constexpr int S = Cf::S;
  constexpr int R = Cf::R;
  constexpr int RB = Cf::RB;
  constexpr int RS = Cf::RS;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;                                              // S stages, 1024-aligned
  uint8_t* rr = ring + S * Cf::STAGE_BYTES;                          // R re-read stages
  float* red = reinterpret_cast<float*>(rr + R * Cf::RR_BYTES);      // [RB][C][TPO][RS] == [RB][128][RS]
  float* hpre = red + RB * kBM * RS;                                 // [RB][128][n]
  float* tot = hpre + RB * kBM * n;                                  // [TPO][RS]  (owner sums)
  float* hp_s = tot + kBM * RS;                                      // [TPO][n]
  uint64_t* bars = reinterpret_cast<uint64_t*>(hp_s + kBM * n);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B::count);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t cid = cluster_id_x();
  const uint32_t ncl = nclusters_x();
  const int C = p.C;
  const int TPO = kBM / C;                 // tokens owned per CTA per tile
  const int D = p.D;
  const int Dc = p.Dc;
  const int DCH = Dc / kBK;                // 64-wide d-chunks per stream in the slice
  const int KB = n * DCH;                  // K-blocks per tile per CTA
  const int nD = n * D;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(bar(B::full + i), 1);
      mbar_init(bar(B::empty + i), 1 + 4);
    }
    for (int i = 0; i < Cf::NBUF; ++i) {
      mbar_init(bar(B::acc_full + i), 1);
      mbar_init(bar(B::acc_empty + i), 4);
    }
    for (int i = 0; i < RB; ++i) {
      mbar_init(bar(B::red_full + i), kBM);
      mbar_init(bar(B::red_free + i), C);
      mbar_init(bar(B::hpre_full + i), kBM);
      mbar_init(bar(B::hpre_free + i), C);
    }
    for (int i = 0; i < R; ++i) {
      mbar_init(bar(B::rr_full + i), 1);
      mbar_init(bar(B::rr_empty + i), 4);
    }
    *abort_flag = 0;
    fence_mbarrier_init_cluster();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cf::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&map_x2d);
    prefetch_tensormap(&map_phi);
    prefetch_tensormap(&map_x3d);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_sync_all();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtx wc{abort_flag, p.status};

  const int my_tiles = (int)cid < p.num_tiles ? (p.num_tiles - 1 - (int)cid) / (int)ncl + 1 : 0;

  // Control flow is identical with or without a timeout: a bounded wait that
  // gives up sets *abort_flag, every later wait of this CTA returns at once,
  // and only the issue of TMA / tcgen05 work is skipped.  So every named
  // barrier, remote arrival and the final cluster barrier are still reached.
  const bool producer = (lane == 0);
  if (warp == 0) {
    // ------------------------------------------------ W0: TMA producer (x, phi)
    if (producer) {
      const uint64_t pol_keep = l2_policy_evict_last();
      uint32_t it = 0;
      for (int j = 0; j < my_tiles; ++j) {
        const int tile = (int)cid + j * (int)ncl;
        // Optional L2 prefetch of the next tile's slice (tuning; off by default:
        // it doubles the L2 footprint between a tile's first read and the h_in
        // re-read, and B200 keeps only ~55 MB of such reuse distance).
        for (int jt = (j == 0 ? 0 : j + 1); MHC_FWD_PREFETCH && jt <= j + 1 && jt < my_tiles; ++jt) {
          const int pt = (int)cid + jt * (int)ncl;
          for (int kb = 0; kb < KB; ++kb) {
            const int i = kb / DCH, dch = kb - i * DCH;
            tma_prefetch_2d(&map_x2d, i * D + (int)rank * Dc + dch * kBK, pt * kBM);
          }
        }
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          mbar_wait(bar(B::empty + s), ((it / S) & 1) ^ 1, wc);
          if (*abort_flag) continue;
          const int i = kb / DCH, dch = kb - i * DCH;
          const int k0 = i * D + (int)rank * Dc + dch * kBK;
          uint8_t* st = ring + s * Cf::STAGE_BYTES;
          mbar_arrive_expect_tx(bar(B::full + s), Cf::STAGE_BYTES);
          tma_load_2d(smem_u32(st), &map_x2d, bar(B::full + s), k0, tile * kBM, pol_keep);
          tma_load_2d(smem_u32(st + Cf::A_BYTES), &map_phi, bar(B::full + s), k0, 0, pol_keep);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ W1: tcgen05.mma issuer
    if (producer) {
      constexpr uint32_t idesc = idesc_bf16_f32(kBM, Cf::NB, false, false);
      uint32_t it = 0, g = 0;
      for (int j = 0; j < my_tiles; ++j) {
        for (int kb = 0; kb < KB; ++kb, ++it, ++g) {
          // one fresh accumulator per K-block
          const int ab = g % Cf::NBUF;
          mbar_wait(bar(B::acc_empty + ab), ((g / Cf::NBUF) & 1) ^ 1, wc);
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + ab * Cf::ACC_COLS;
          const int s = it % S;
          mbar_wait(bar(B::full + s), (it / S) & 1, wc);
          tc_fence_after();
          if (*abort_flag) continue;
          uint8_t* st = ring + s * Cf::STAGE_BYTES;
          const uint64_t a0 = desc_kmajor_sw128(smem_u32(st));
          const uint64_t b0 = desc_kmajor_sw128(smem_u32(st + Cf::A_BYTES));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) umma_bf16(d_tmem, a0 + 2 * kk, b0 + 2 * kk, idesc, kk != 0);
          umma_commit(bar(B::empty + s));
          umma_commit(bar(B::acc_full + ab));
        }
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------ W2: TMA producer (L2 re-read for h_in)
    if (producer) {
      const uint64_t pol_drop = l2_policy_evict_first();
      uint32_t it = 0;
      for (int j = 0; j < my_tiles; ++j) {
        const int tile = (int)cid + j * (int)ncl;
        for (int sub = 0; sub < kBM / Cf::RR_TOK; ++sub) {
          for (int dch = 0; dch < DCH; ++dch, ++it) {
            const int r = it % R;
            mbar_wait(bar(B::rr_empty + r), ((it / R) & 1) ^ 1, wc);
            if (*abort_flag) continue;
            mbar_arrive_expect_tx(bar(B::rr_full + r), Cf::RR_BYTES);
            tma_load_3d(smem_u32(rr + r * Cf::RR_BYTES), &map_x3d, bar(B::rr_full + r),
                        (int)rank * Dc + dch * kBK, 0, tile * kBM + sub * Cf::RR_TOK, pol_drop);
          }
        }
      }
    }
  } else if (warp < 7) {
    // ------------------------------------------------ WG_SR: sum x^2 + fold accumulators, send to owner
    const int q = warp & 3;                   // TMEM lane quadrant of this warp
    const int row = 32 * q + lane;            // token row of the tile = TMEM lane = smem row
    uint32_t it = 0, g = 0;
    constexpr int LAG = 2;                    // fold K-block kb-LAG while reading stage kb
    static_assert(LAG < Cf::NBUF, "accumulator ring shorter than the fold lag");
    // Fold accumulator ring slot of K-block counter gg (NT split terms of each
    // output) into part; narrow outputs sum the block's terms (smallest first)
    // before adding, wide outputs fold in place to stay in registers.
    auto fold = [&](uint32_t gg, float (&part)[N_OUT]) {
      const int ab = gg % Cf::NBUF;
      mbar_wait(bar(B::acc_full + ab), (gg / Cf::NBUF) & 1, wc);
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + ab * Cf::ACC_COLS;
      constexpr bool kBlockSum = N_OUT <= 32;
      float blk[kBlockSum ? N_OUT : 1];
#pragma unroll
      for (int jj = 0; jj < (kBlockSum ? N_OUT : 1); ++jj) blk[jj] = 0.f;
#pragma unroll
      for (int c16 = Cf::NB / 16 - 1; c16 >= 0; --c16) {
        float v[16];
        tmem_ld16(taddr + c16 * 16, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 15; e >= 0; --e) {
          const int col = c16 * 16 + e;
          if (col < Cf::NT * N_OUT) {
            if constexpr (kBlockSum) blk[col % N_OUT] += v[e];
            else part[col % N_OUT] += v[e];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B::acc_empty + ab));
      if constexpr (kBlockSum) {
#pragma unroll
        for (int jj = 0; jj < N_OUT; ++jj) part[jj] += blk[jj];
      }
    };
    for (int j = 0; j < my_tiles; ++j) {
      float part[N_OUT];
#pragma unroll
      for (int jj = 0; jj < N_OUT; ++jj) part[jj] = 0.f;
      float sq = 0.f;
      const uint32_t g0 = g;
      for (int kb = 0; kb < KB; ++kb, ++it, ++g) {
        const int s = it % S;
        mbar_wait(bar(B::full + s), (it / S) & 1, wc);
        {
          const uint32_t base = smem_u32(ring + s * Cf::STAGE_BYTES) + row * 128;
          float c8[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float f[8];
            bf16x8_to_f32(lds128(base + (((c + row) & 7) << 4)), f);
            const float a = fmaf(f[0], f[0], f[1] * f[1]) + fmaf(f[2], f[2], f[3] * f[3]);
            const float b = fmaf(f[4], f[4], f[5] * f[5]) + fmaf(f[6], f[6], f[7] * f[7]);
            c8[c] = a + b;
          }
          sq += ((c8[0] + c8[1]) + (c8[2] + c8[3])) + ((c8[4] + c8[5]) + (c8[6] + c8[7]));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B::empty + s));
        if (kb >= LAG) fold(g - LAG, part);
      }
      for (uint32_t gg = (g - g0 >= LAG ? g - LAG : g0); gg < g; ++gg) fold(gg, part);
      // send (part, sq) of token `row` to its owner CTA
      const int rb = j % RB;
      const uint32_t rph = (j / RB) & 1;
      mbar_wait<true>(bar(B::red_free + rb), rph ^ 1, wc);
      const int owner = row / TPO;
      const uint32_t local = smem_u32(red + (rb * kBM + (int)rank * TPO + (row % TPO)) * RS);
      const uint32_t dst = mapa_shared(local, owner);
#pragma unroll
      for (int jj = 0; jj + 4 <= N_OUT + 1; jj += 4) {
        const float v3 = (jj + 3 < N_OUT) ? part[jj + 3] : sq;
        st_cluster_v4_f32(dst + 4 * jj, part[jj], part[jj + 1], part[jj + 2], v3);
      }
#pragma unroll
      for (int jj = (N_OUT + 1) / 4 * 4; jj < N_OUT + 1; ++jj) st_cluster_f32(dst + 4 * jj, jj < N_OUT ? part[jj] : sq);
      mbar_arrive_remote(bar(B::red_full + rb), owner);
    }
  } else if (warp < 11) {
    // ------------------------------------------------ WG_A: owner reduction -> gates -> h_pre broadcast
    const int tid = threadIdx.x - 7 * 32;     // 0..127
    const float a_pre = p.alpha[0], a_post = p.alpha[1], a_res = p.alpha[2];
    for (int j = 0; j < my_tiles; ++j) {
      const int tile = (int)cid + j * (int)ncl;
      const int rb = j % RB;
      const uint32_t rph = (j / RB) & 1;
      // (4) owner: fixed-order sum over the C partials of my TPO tokens
      mbar_wait<true>(bar(B::red_full + rb), rph, wc);
      for (int idx = tid; idx < TPO * (N_OUT + 1); idx += 128) {
        const int lt = idx / (N_OUT + 1), jj = idx - lt * (N_OUT + 1);
        float sum = 0.f;
        for (int src = 0; src < C; ++src) sum += red[(rb * kBM + src * TPO + lt) * RS + jj];
        tot[lt * RS + jj] = sum;
      }
      named_sync(1, 128);
      if (tid < C) mbar_arrive_remote(bar(B::red_free + rb), tid);   // one release per destination CTA
      // (5) outputs of my tokens
      const float inv_nd = 1.0f / (float)nD;
      for (int idx = tid; idx < TPO * N_OUT; idx += 128) {
        const int lt = idx / N_OUT, jj = idx - lt * N_OUT;
        const int64_t t = (int64_t)tile * kBM + (int)rank * TPO + lt;
        const float ir = 1.0f / sqrtf(tot[lt * RS + N_OUT] * inv_nd + p.norm_eps);
        const float hm = tot[lt * RS + jj];
        const float v = hm * ir;
        if (jj < n) {
          const float hp = sigmoid_acc(a_pre * v + p.bias[jj]) + p.hc_eps;
          hp_s[lt * n + jj] = hp;
          if (t < p.T && p.h_pre) p.h_pre[t * n + jj] = hp;
        } else if (jj < 2 * n) {
          if (t < p.T) p.h_post[t * n + (jj - n)] = 2.0f * sigmoid_acc(a_post * v + p.bias[jj]);
        } else {
          if (t < p.T) p.h_res[t * (n * n) + (jj - 2 * n)] = a_res * v + p.bias[jj];
        }
        if (t < p.T) {
          if (p.h_mix) p.h_mix[t * N_OUT + jj] = hm;
          if (jj == 0 && p.inv_rms) p.inv_rms[t] = ir;
        }
      }
      named_sync(1, 128);
      // (6) broadcast h_pre of my tokens to every CTA of the cluster
      mbar_wait<true>(bar(B::hpre_free + rb), rph ^ 1, wc);
      for (int idx = tid; idx < TPO * C; idx += 128) {
        const int lt = idx % TPO, dstc = idx / TPO;
        const uint32_t local = smem_u32(hpre + (rb * kBM + (int)rank * TPO + lt) * n);
        const uint32_t dst = mapa_shared(local, dstc);
#pragma unroll
        for (int i = 0; i < n; ++i) st_cluster_f32(dst + 4 * i, hp_s[lt * n + i]);
        mbar_arrive_remote(bar(B::hpre_full + rb), dstc);
      }
      named_sync(1, 128);
    }
  } else {
    // ------------------------------------------------ WG_B: h_in of this CTA's d-slice
    const int tid = threadIdx.x - 11 * 32;    // 0..127
    const uint64_t pol_out = l2_policy_evict_first();   // h_in must not push out data awaiting re-read
    uint32_t it = 0;
    for (int j = 0; j < my_tiles; ++j) {
      const int tile = (int)cid + j * (int)ncl;
      const int rb = j % RB;
      mbar_wait<true>(bar(B::hpre_full + rb), (j / RB) & 1, wc);
      for (int sub = 0; sub < kBM / Cf::RR_TOK; ++sub) {
        for (int dch = 0; dch < DCH; ++dch, ++it) {
          const int r = it % R;
          mbar_wait(bar(B::rr_full + r), (it / R) & 1, wc);
          const uint32_t base = smem_u32(rr + r * Cf::RR_BYTES);
          for (int task = tid; task < Cf::RR_TOK * 8; task += 128) {
            const int t = task >> 3, c = task & 7;
            const int trow = sub * Cf::RR_TOK + t;
            float acc[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
            for (int i = 0; i < n; ++i) {
              const float hp = hpre[(rb * kBM + trow) * n + i];
              float f[8];
              bf16x8_to_f32(lds128(base + ((t * n + i) << 7) + (c << 4)), f);
#pragma unroll
              for (int e = 0; e < 8; ++e) acc[e] = fmaf(hp, f[e], acc[e]);
            }
            const int64_t tok = (int64_t)tile * kBM + trow;
            if (tok < p.T) {
              uint4 o;
              o.x = pack_bf16x2(acc[0], acc[1]);
              o.y = pack_bf16x2(acc[2], acc[3]);
              o.z = pack_bf16x2(acc[4], acc[5]);
              o.w = pack_bf16x2(acc[6], acc[7]);
              st_global_hint(p.h_in + tok * D + (int)rank * Dc + dch * kBK + c * 8, o, pol_out);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B::rr_empty + r));
        }
      }
      named_sync(2, 128);
      if (tid < C) mbar_arrive_remote(bar(B::hpre_free + rb), tid);
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cf::TMEM_COLS);
  }
  cluster_sync_all();
}

// phi [N_OUT, nD] f32 -> phis [NB, nD] bf16: rows t*N_OUT + j hold the t-th
// bf16 term of phi[j] (hi, mid, lo: each term rounds what the previous ones
// left), rows >= NT*N_OUT are zero.
template <int n>
__global__ void __launch_bounds__(256) split_phi_kernel(const float* __restrict__ phi, uint16_t* __restrict__ phis,
                                                        int nD) {
  // phis [NB][nD]: row term*N_OUT + j holds bf16 term `term` of phi[j]; rows
  // past NT*N_OUT are zero.  Each thread writes 8 consecutive k (one 16-byte
  // store); needs nD % 8 == 0.
  using Cf = Cfg<n>;
  const int64_t per_row = nD / 8;
  const int64_t total = (int64_t)Cf::NB * per_row;
  for (int64_t idx = blockIdx.x * 256ll + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * 256) {
    const int r = (int)(idx / per_row);
    const int64_t k = (idx - (int64_t)r * per_row) * 8;
    uint32_t w[4] = {0, 0, 0, 0};
    if (r < Cf::NT * Cf::N_OUT) {
      const int term = r / Cf::N_OUT, j = r - term * Cf::N_OUT;
      const float4 a = __ldg(reinterpret_cast<const float4*>(phi + (int64_t)j * nD + k));
      const float4 b = __ldg(reinterpret_cast<const float4*>(phi + (int64_t)j * nD + k + 4));
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        uint32_t t2[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          float rem = v[2 * h + q];
          uint16_t o = 0;
          for (int tt = 0; tt <= term; ++tt) {
            o = f32_to_bf16_bits(rem);
            rem -= bf16_bits_to_f32(o);
          }
          t2[q] = o;
        }
        w[h] = t2[0] | (t2[1] << 16);
      }
    }
    *reinterpret_cast<uint4*>(phis + (int64_t)r * nD + k) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace fwdtc
}  // namespace mhc
