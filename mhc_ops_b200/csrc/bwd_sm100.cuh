// Backward of the mHC pre-op on sm_100a: cluster K-split, tcgen05 GEMMs.
//
// Math: src/backward/golden.py:38-96.  Per token t (row of x):
//   dh_pre[i] = sum_d dh_in[d] x[i,d]                                  (:51)
//   dh_mix    = [a_pre dh_pre2, a_post dh_post2, a_res dh_res] * inv_rms (:53-62)
//   c         = (sum_j dh_mix_tmp[j] h_mix[j]) inv_rms^3 / nD           (:74, :89)
//   dx[k]     = gamma[k] (dh_mix @ phi)[k] - c x[k] + h_pre[i] dh_in[d] (:65, :89-94)
// and over tokens: G = dh_mix^T x, dphi = G * gamma (:68-69), dgamma[k] =
// sum_j phi[j,k] G[j,k] (= sum_t x dvecX_mm, :93), dalpha (:77-80), dbias (:83-86).
//
// A cluster of C CTAs owns one 128-token tile at a time; CTA r owns the
// d-slice [r*Dc, (r+1)*Dc) of every stream.  Per tile:
//   * WG_P (4 warps, phase 1) reads x and dh_in of its slice straight from HBM
//     (warp per token, L2 evict-last), forms the partial dh_pre of each token,
//     sends it to the token's owner CTA (DSMEM); the owner reduces the C
//     partials in rank order, computes dh_mix, c, the dalpha/dbias terms and
//     broadcasts one record per token (dh_mix, c, h_pre) to every CTA.
//   * W0 re-reads the slice through L2 with TMA (x blocks [128 tok x 64 k],
//     dh_in blocks, 128-B swizzle, evict-first); W2 streams pre-laid-out
//     split-phi images (1-D bulk copies, 3 bf16 terms of phi per k);
//   * WG_E (4 warps) turns the records into the UMMA operand DHM [128 tok x
//     3 segments]: the 3 bf16 terms (hi, mid, lo) of dh_mix, each segment
//     padded to a multiple of 16;
//   * W1 issues tcgen05.mma: dvecX = sum over 6 (dh term, phi term) products
//     (smallest first: m.M, l.H, h.L, m.H, h.M, h.H; exact to ~2^-23 in the
//     fp32 sum) per 64-k block (M=128 tok, N=64, K=segment) and
//     G += x^T . DHM (M=128 k, N=segment, K=3x128 tokens; x read MN-major
//     straight from two adjacent TMA stages, DHM read MN-major);
//   * WG_E reads dvecX (TMEM lane = token) and writes dx; every FT tiles it
//     flushes G from TMEM into the per-cluster partial (single writer per
//     address, fixed order).
#pragma once

#include "common.cuh"
#include "sm100.cuh"

// Optional per-tile timestamp hook (a profiling build defines it); no-op here.
#ifndef MHC_BWD_TRACE
#define MHC_BWD_TRACE(slot) ((void)0)
#endif
#ifndef MHC_BWD_TRACE_Q
#define MHC_BWD_TRACE_Q(slot) ((void)0)
#endif
// Tiles of look-ahead for an L2 prefetch of the next tiles' slices (tuning;
// off: on B200 data survives in L2 only for ~55 MB of intervening traffic, and
// a whole-tile prefetch pushes the phase-2 re-reads past that distance).
#ifndef MHC_BWD_PREFETCH
#define MHC_BWD_PREFETCH 0
#endif
// Phase-2 stages of look-ahead for the producer's L2 prefetch (tuning; 0 = off).
#ifndef MHC_BWD_PF_STAGES
#define MHC_BWD_PF_STAGES 0
#endif

namespace mhc {
namespace bwdtc {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kWarpE0 = 7;          // first epilogue warp
constexpr int kThreadsE = 8 * 32;   // WG_E: 8 warps
constexpr int kThreads = kWarpE0 * 32 + kThreadsE;   // W0, W1, W2, WG_P(4), WG_E(8)
constexpr int kSmemLimit = 232448;

constexpr int round_up(int v, int a) { return (v + a - 1) / a * a; }

template <int n>
struct Cfg {
  static constexpr int N_OUT = n * n + 2 * n;
  static constexpr int SEGW = round_up(N_OUT, 16);       // one split-term segment (N of G)
  static constexpr int KA = 3 * SEGW;                    // DHM / phi-image row: 3 term segments
  static constexpr int RG_BYTES = (KA / 8) * 128;        // one 8-row group of a K-major interleaved image
  static constexpr int PH_BYTES = 8 * RG_BYTES;          // split-phi image of one 64-k block
  static constexpr int DHM_BYTES = 16 * RG_BYTES;        // 128 token rows
  static constexpr int NG = SEGW;                        // G accumulator columns
  static constexpr int X_BYTES = kBM * 128;
  static constexpr int XS = 4;                           // x ring (2 adjacent pairs)
  static constexpr int DS = 2;
  static constexpr int PS = 3;
  static constexpr int RECW = round_up(N_OUT + 1 + n, 4);
  static constexpr int RB = 2;                           // dh_pre exchange buffers
  static constexpr int MAX_TPO = 32;                     // C >= 4
  static constexpr int MAX_KC = 1792;                    // d-slice * n per CTA
  static constexpr int CW = 3 + N_OUT;                   // dalpha / dbias columns
  // owner inputs per token: h_mix[N_OUT], h_pre[n], h_post[n], dh_post[n], dh_res[n*n], inv_rms
  static constexpr int OWN_IN = N_OUT + 3 * n + n * n + 1;
  static constexpr int OWNW = round_up(OWN_IN, 4);

  static constexpr int smem_bytes() {
    return 1024 + XS * X_BYTES + DS * X_BYTES + PS * PH_BYTES + DHM_BYTES + X_BYTES /*dx staging*/ +
           MAX_KC * 4 /*gamma slice*/ + RB * kBM * n * 4 /*pdh*/ + kBM * RECW * 4 /*bc*/ +
           MAX_TPO * (n + RECW + CW + OWNW) * 4 /*owner scratch*/ + 512;
  }
  static constexpr int SMEM = smem_bytes();
  static_assert(SMEM <= kSmemLimit, "backward tile does not fit in shared memory");
  static_assert(n % 2 == 0, "G pairs two streams of a d-chunk");
};

struct Params {
  const uint16_t* x;
  const uint16_t* dh_in;
  const float* alpha;
  const float* inv_rms;
  const float* h_mix;
  const float* h_pre;
  const float* h_post;
  const float* dh_post;
  const float* dh_res;
  const float* gamma;     // may be null
  const uint8_t* phit;    // split-phi images, PH_BYTES per 64-k block
  uint16_t* dx;
  float* gpart;           // [num_clusters][N_OUT][nD]
  float* abpart;          // [num_clusters * C][3 + N_OUT]
  int* status;
  int64_t T;
  int D;
  int Dc;
  int C;
  int num_tiles;
  int FT;                 // tiles per G flush
  int dv_bufs;            // 1 or 2 dvecX TMEM buffers
  float hc_eps;
};

template <int n>
struct Bars {
  using Cf = Cfg<n>;
  static constexpr int x_full = 0;
  static constexpr int x_empty = x_full + Cf::XS;
  static constexpr int dh_full = x_empty + Cf::XS;
  static constexpr int dh_empty = dh_full + Cf::DS;
  static constexpr int ph_full = dh_empty + Cf::DS;
  static constexpr int ph_empty = ph_full + Cf::PS;
  static constexpr int dv_full = ph_empty + Cf::PS;
  static constexpr int dv_empty = dv_full + 2;
  static constexpr int dhm_full = dv_empty + 2;
  static constexpr int dhm_free = dhm_full + 1;
  static constexpr int g_full = dhm_free + 1;
  static constexpr int g_empty = g_full + 1;
  static constexpr int p_full = g_empty + 1;
  static constexpr int p_free = p_full + Cf::RB;
  static constexpr int bc_full = p_free + Cf::RB;
  static constexpr int bc_free = bc_full + 1;
  static constexpr int count = bc_free + 1;
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

__device__ __forceinline__ uint4 ldg_keep(const void* ptr, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(ptr), "l"(pol));
  return v;
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                          uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// smem -> global tiled TMA store (out-of-range rows of the box are not written)
// with an L2 eviction-priority hint.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int32_t c0, int32_t c1,
                                             uint64_t policy) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "l"(policy)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void red_add_f32(float* addr, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
}

// K-major operand without swizzle: 8x16-byte core matrices, LBO between
// K-adjacent cores, SBO between 8-row groups.
__device__ __forceinline__ uint64_t desc_kmajor_interleave(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;   // layout type 0 = no swizzle
}

// Byte offset of element (row, kk) in a K-major interleaved image whose
// 8-row groups are sbo bytes apart.
__device__ __forceinline__ uint32_t interleave_off(int row, int kk, int sbo) {
  return (uint32_t)((row >> 3) * sbo + (kk >> 3) * 128 + (row & 7) * 16 + (kk & 7) * 2);
}

// The six (dh_mix term, phi term) products of dvecX, smallest first:
// m.M, l.H, h.L, m.H, h.M, h.H (term 0 = hi, 1 = mid, 2 = lo).
__device__ __forceinline__ int prod_a_term(int pr) { return pr == 0 ? 1 : pr == 1 ? 2 : pr == 3 ? 1 : 0; }
__device__ __forceinline__ int prod_b_term(int pr) { return pr == 0 ? 1 : pr == 2 ? 2 : pr == 4 ? 1 : 0; }

// t-th bf16 term of v (0 = hi, 1 = mid, 2 = lo): each rounds what is left.
__device__ __forceinline__ uint16_t split_term(float v, int term) {
  uint16_t out = 0;
  for (int tt = 0; tt <= term; ++tt) {
    out = f32_to_bf16_bits(v);
    v -= bf16_bits_to_f32(out);
  }
  return out;
}

template <int n>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_kernel(const __grid_constant__ CUtensorMap map_x2d, const __grid_constant__ CUtensorMap map_dh,
               const __grid_constant__ CUtensorMap map_dx, const Params p) {
  using Cf = Cfg<n>;
  using B = Bars<n>;
  constexpr int N_OUT = Cf::N_OUT;
  constexpr int RECW = Cf::RECW;
  constexpr int RB = Cf::RB;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xr = smem;                                  // XS x blocks (pairs adjacent)
  uint8_t* dhr = xr + Cf::XS * Cf::X_BYTES;            // DS dh_in blocks
  uint8_t* phr = dhr + Cf::DS * Cf::X_BYTES;           // PS split-phi images
  uint8_t* dhm = phr + Cf::PS * Cf::PH_BYTES;          // dh_mix terms: A of dvecX, B of G
  uint8_t* dxs = dhm + Cf::DHM_BYTES;                  // dx staging [128 tok x 64] (128-B swizzle)
  float* gam_s = reinterpret_cast<float*>(dxs + Cf::X_BYTES);       // [n][Dc] gamma slice
  float* pdh = gam_s + Cf::MAX_KC;                     // [RB][128][n]
  float* bc = pdh + RB * kBM * n;                      // [128][RECW]
  float* dhp_s = bc + kBM * RECW;                      // [TPO][n]
  float* rec_s = dhp_s + Cf::MAX_TPO * n;              // [TPO][RECW]
  float* contrib = rec_s + Cf::MAX_TPO * RECW;         // [TPO][CW]: dalpha (3), dbias (N_OUT) terms
  float* own_in = contrib + Cf::MAX_TPO * Cf::CW;      // [TPO][OWNW] owner inputs of this tile
  uint64_t* bars = reinterpret_cast<uint64_t*>(own_in + Cf::MAX_TPO * Cf::OWNW);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B::count);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t cid = cluster_id_x();
  const uint32_t ncl = nclusters_x();
  const int C = p.C;
  const int TPO = kBM / C;
  const int D = p.D;
  const int Dc = p.Dc;
  const int DCH = Dc / kBK;
  const int nD = n * D;
  const int KC = n * Dc;
  const int NPAIR = KC / 128;                 // G blocks of 128 k per CTA
  const int DVB = p.dv_bufs;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  // gamma slice of this CTA: gam_s[i*Dc + dd] = gamma[i*D + rank*Dc + dd]
  for (int idx = threadIdx.x; idx < KC; idx += kThreads) {
    const int i = idx / Dc, dd = idx - i * Dc;
    gam_s[idx] = p.gamma ? p.gamma[(int64_t)i * D + (int64_t)rank * Dc + dd] : 1.0f;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < Cf::XS; ++i) {
      mbar_init(bar(B::x_full + i), 1);
      mbar_init(bar(B::x_empty + i), 1 + kThreadsE / 32);
    }
    for (int i = 0; i < Cf::DS; ++i) {
      mbar_init(bar(B::dh_full + i), 1);
      mbar_init(bar(B::dh_empty + i), kThreadsE / 32);
    }
    for (int i = 0; i < Cf::PS; ++i) {
      mbar_init(bar(B::ph_full + i), 32);   // one cp.async arrival per lane of W2
      mbar_init(bar(B::ph_empty + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B::dv_full + i), 1);
      mbar_init(bar(B::dv_empty + i), kThreadsE / 32);
    }
    mbar_init(bar(B::dhm_full), kThreadsE);
    mbar_init(bar(B::dhm_free), 1);
    mbar_init(bar(B::g_full), 1);
    mbar_init(bar(B::g_empty), kThreadsE / 32);
    for (int i = 0; i < RB; ++i) {
      mbar_init(bar(B::p_full + i), kBM);
      mbar_init(bar(B::p_free + i), C);
    }
    mbar_init(bar(B::bc_full), kBM);
    mbar_init(bar(B::bc_free), C);
    *abort_flag = 0;
    fence_mbarrier_init_cluster();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&map_x2d);
    prefetch_tensormap(&map_dh);
    prefetch_tensormap(&map_dx);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_sync_all();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_dv = tmem_base;                       // DVB x 64 columns
  const uint32_t tmem_g = tmem_base + DVB * 64;             // NPAIR x NG columns
  const WaitCtx wc{abort_flag, p.status};
  const int my_tiles = (int)cid < p.num_tiles ? (p.num_tiles - 1 - (int)cid) / (int)ncl + 1 : 0;
  const bool producer = (lane == 0);

  if (warp == 0) {
    // ------------------------------------------------ W0: TMA producer (phase-2 re-read)
    if (producer) {
      const uint64_t pol_drop = l2_policy_evict_first();
      uint32_t q = 0, dq = 0;
      for (int j = 0; j < my_tiles; ++j) {
        const int tile = (int)cid + j * (int)ncl;
        for (int dch = 0; dch < DCH; ++dch, ++dq) {
          const int ds = dq % Cf::DS;
          mbar_wait(bar(B::dh_empty + ds), ((dq / Cf::DS) & 1) ^ 1, wc);
          MHC_BWD_TRACE_Q(1);
          if (!*abort_flag) {
            mbar_arrive_expect_tx(bar(B::dh_full + ds), Cf::X_BYTES);
            tma_load_2d(smem_u32(dhr + ds * Cf::X_BYTES), &map_dh, bar(B::dh_full + ds), (int)rank * Dc + dch * kBK,
                        tile * kBM, pol_drop);
          }
          for (int i = 0; i < n; ++i, ++q) {
            const int s = q % Cf::XS;
            const int k0 = i * D + (int)rank * Dc + dch * kBK;
            if (MHC_BWD_PF_STAGES > 0) {
              // stage q + PF of this CTA's (tile, dch, i) sequence
              const int qa = (dch * n + i) + MHC_BWD_PF_STAGES;
              const int jt = j + qa / (DCH * n), r2 = qa % (DCH * n);
              if (jt < my_tiles) {
                const int pd = r2 / n, pi = r2 % n;
                const int pt = (int)cid + jt * (int)ncl;
                tma_prefetch_2d(&map_x2d, pi * D + (int)rank * Dc + pd * kBK, pt * kBM);
                if (pi == 0) tma_prefetch_2d(&map_dh, (int)rank * Dc + pd * kBK, pt * kBM);
              }
            }
            mbar_wait(bar(B::x_empty + s), ((q / Cf::XS) & 1) ^ 1, wc);
            MHC_BWD_TRACE_Q(0);
            if (dch == 0 && i == 0) MHC_BWD_TRACE(11);
            if (dch == DCH - 1 && i == n - 1) MHC_BWD_TRACE(12);
            if (!*abort_flag) {
              mbar_arrive_expect_tx(bar(B::x_full + s), Cf::X_BYTES);
              tma_load_2d(smem_u32(xr + s * Cf::X_BYTES), &map_x2d, bar(B::x_full + s), k0, tile * kBM, pol_drop);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ W1: tcgen05.mma issuer
    if (producer) {
      constexpr uint32_t idesc_dv = idesc_bf16_f32(kBM, kBK, false, false);
      constexpr uint32_t idesc_g = idesc_bf16_f32(kBM, Cf::NG, true, true);
      uint32_t q = 0, flushes = 0;
      for (int j = 0; j < my_tiles; ++j) {
        mbar_wait(bar(B::dhm_full), j & 1, wc);
        MHC_BWD_TRACE(9);
        tc_fence_after();
        const bool g_restart = (j % p.FT) == 0;
        if (g_restart && j > 0) {
          mbar_wait(bar(B::g_empty), (flushes - 1) & 1, wc);   // previous G group read out
          tc_fence_after();
        }
        for (int dch = 0; dch < DCH; ++dch) {
          for (int i = 0; i < n; ++i, ++q) {
            const int s = q % Cf::XS;
            const int ps = q % Cf::PS;
            const int dvb = DVB == 2 ? (int)(q & 1) : 0;
            const uint32_t dvph = DVB == 2 ? (q >> 1) & 1 : q & 1;
            mbar_wait(bar(B::ph_full + ps), (q / Cf::PS) & 1, wc);
            mbar_wait(bar(B::dv_empty + dvb), dvph ^ 1, wc);
            MHC_BWD_TRACE_Q(3);
            tc_fence_after();
            if (!*abort_flag) {
              const uint32_t dhm_a = smem_u32(dhm), ph_a = smem_u32(phr + ps * Cf::PH_BYTES);
#pragma unroll
              for (int pr = 0; pr < 6; ++pr) {
#pragma unroll
                for (int ks = 0; ks < Cf::SEGW / 16; ++ks) {
                  const uint32_t ca = (prod_a_term(pr) * Cf::SEGW + ks * 16) * 16;
                  const uint32_t cb = (prod_b_term(pr) * Cf::SEGW + ks * 16) * 16;
                  umma_bf16(tmem_dv + dvb * 64, desc_kmajor_interleave(dhm_a + ca, 128, Cf::RG_BYTES),
                            desc_kmajor_interleave(ph_a + cb, 128, Cf::RG_BYTES), idesc_dv, pr != 0 || ks != 0);
                }
              }
              umma_commit(bar(B::ph_empty + ps));
              umma_commit(bar(B::dv_full + dvb));
            }
            if (i & 1) {
              // G over the pair of stages (s-1, s): rows 0..63 stream i-1, 64..127 stream i
              mbar_wait(bar(B::x_full + s - 1), ((q - 1) / Cf::XS) & 1, wc);
              mbar_wait(bar(B::x_full + s), (q / Cf::XS) & 1, wc);
              MHC_BWD_TRACE_Q(4);
              tc_fence_after();
              if (!*abort_flag) {
                const int blk = dch * (n / 2) + i / 2;
                const uint32_t xa = smem_u32(xr + (s - 1) * Cf::X_BYTES);
                const uint32_t ga = smem_u32(dhm);
#pragma unroll 1
                for (int e = 2; e >= 0; --e) {            // lo, mid, hi terms of dh_mix
#pragma unroll
                  for (int ks = 0; ks < kBM / 16; ++ks) {
                    const uint64_t ad = desc_mnmajor_sw128(xa + ks * 2048, Cf::X_BYTES, 1024);
                    // DHM read MN-major: N = the SEGW columns of term e, K = tokens
                    const uint64_t bd =
                        desc_kmajor_interleave(ga + e * Cf::SEGW * 16 + ks * 2 * Cf::RG_BYTES, Cf::RG_BYTES, 128);
                    umma_bf16(tmem_g + blk * Cf::NG, ad, bd, idesc_g, !(g_restart && e == 2 && ks == 0));
                  }
                }
                umma_commit(bar(B::x_empty + s - 1));
                umma_commit(bar(B::x_empty + s));
              }
            }
          }
        }
        MHC_BWD_TRACE(10);
        if (!*abort_flag) umma_commit(bar(B::dhm_free));
        if ((j + 1) % p.FT == 0 || j == my_tiles - 1) {
          if (!*abort_flag) umma_commit(bar(B::g_full));
          ++flushes;
        }
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------ W2: split-phi image producer
    // The whole warp copies each image with 16-byte cp.async (LSU path), so the
    // TMA engine only carries x, dh_in and the dx stores.
    uint32_t q = 0;
    for (int j = 0; j < my_tiles; ++j) {
      for (int dch = 0; dch < DCH; ++dch) {
        for (int i = 0; i < n; ++i, ++q) {
          const int ps = q % Cf::PS;
          const int k0 = i * D + (int)rank * Dc + dch * kBK;
          mbar_wait(bar(B::ph_empty + ps), ((q / Cf::PS) & 1) ^ 1, wc);
          if (lane == 0) MHC_BWD_TRACE_Q(2);
          if (!*abort_flag) {
            const uint8_t* src = p.phit + (size_t)(k0 / kBK) * Cf::PH_BYTES;
            const uint32_t dst = smem_u32(phr + ps * Cf::PH_BYTES);
#pragma unroll 4
            for (int off = lane * 16; off < Cf::PH_BYTES; off += 32 * 16) cp_async16(dst + off, src + off);
          }
          cp_async_arrive_noinc(bar(B::ph_full + ps));   // fires when this lane's copies have landed
        }
      }
    }
  } else if (warp < 7) {
    // ------------------------------------------------ WG_P: phase 1 (dh_pre partials) + owner + broadcast
    const int tid = threadIdx.x - 3 * 32;    // 0..127
    const int wp = warp - 3;                 // 0..3, 32 token rows each
    const uint64_t pol_keep = l2_policy_evict_last();
    const float a_pre = p.alpha[0], a_post = p.alpha[1], a_res = p.alpha[2];
    const float inv_nd = 1.0f / (float)nD;
    float ab_acc = 0.f;                      // thread c < 3+N_OUT: running dalpha/dbias column
    for (int j = 0; j < my_tiles; ++j) {
      const int tile = (int)cid + j * (int)ncl;
      if (tid == 0) MHC_BWD_TRACE(0);
      // Pull the slice of the tile after this one into L2 now (tile 0 too, at
      // the start), so phase-1 loads see L2 latency and phase 2 re-reads hit.
      if (tid == 0 && MHC_BWD_PREFETCH > 0) {
        for (int jt = (j == 0 ? 0 : j + MHC_BWD_PREFETCH); jt <= j + MHC_BWD_PREFETCH && jt < my_tiles; ++jt) {
          const int pt = (int)cid + jt * (int)ncl;
          for (int dch = 0; dch < DCH; ++dch) {
            tma_prefetch_2d(&map_dh, (int)rank * Dc + dch * kBK, pt * kBM);
            for (int i = 0; i < n; ++i) tma_prefetch_2d(&map_x2d, i * D + (int)rank * Dc + dch * kBK, pt * kBM);
          }
        }
      }
      // (0) small per-token inputs of the tokens this CTA owns, loaded in
      // parallel now so the owner step reads them from smem.  own_in is free:
      // the previous tile's owner step finished before its last named barrier.
      for (int idx = tid; idx < TPO * Cf::OWN_IN; idx += 128) {
        const int lt = idx / Cf::OWN_IN, f = idx - lt * Cf::OWN_IN;
        const int64_t t = (int64_t)tile * kBM + (int)rank * TPO + lt;
        float v = 0.f;
        if (t < p.T) {
          if (f < N_OUT) v = __ldg(p.h_mix + t * N_OUT + f);
          else if (f < N_OUT + n) v = __ldg(p.h_pre + t * n + (f - N_OUT));
          else if (f < N_OUT + 2 * n) v = __ldg(p.h_post + t * n + (f - N_OUT - n));
          else if (f < N_OUT + 3 * n) v = __ldg(p.dh_post + t * n + (f - N_OUT - 2 * n));
          else if (f < N_OUT + 3 * n + n * n) v = __ldg(p.dh_res + t * (n * n) + (f - N_OUT - 3 * n));
          else v = __ldg(p.inv_rms + t);
        }
        own_in[lt * Cf::OWNW + f] = v;
      }
      // (1) partial dh_pre of this warp's 32 tokens over the CTA's d-slice
      float mine[n];
#pragma unroll
      for (int i = 0; i < n; ++i) mine[i] = 0.f;
      for (int tt = 0; tt < 32; tt += 4) {
        float acc[4][n];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int i = 0; i < n; ++i) acc[u][i] = 0.f;
        for (int e0 = lane * 8; e0 < Dc; e0 += 256) {
          uint4 g[4], xv[4][n];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int64_t t = (int64_t)tile * kBM + wp * 32 + tt + u;
            if (t < p.T) {
              g[u] = ldg_keep(p.dh_in + t * D + (int64_t)rank * Dc + e0, pol_keep);
#pragma unroll
              for (int i = 0; i < n; ++i)
                xv[u][i] = ldg_keep(p.x + t * nD + (int64_t)i * D + (int64_t)rank * Dc + e0, pol_keep);
            } else {
              g[u] = make_uint4(0, 0, 0, 0);
#pragma unroll
              for (int i = 0; i < n; ++i) xv[u][i] = make_uint4(0, 0, 0, 0);
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float gf[8];
            bf16x8_to_f32(g[u], gf);
#pragma unroll
            for (int i = 0; i < n; ++i) {
              float xf[8];
              bf16x8_to_f32(xv[u][i], xf);
              float s0 = gf[0] * xf[0], s1 = gf[1] * xf[1];
              s0 = fmaf(gf[2], xf[2], s0);
              s1 = fmaf(gf[3], xf[3], s1);
              s0 = fmaf(gf[4], xf[4], s0);
              s1 = fmaf(gf[5], xf[5], s1);
              s0 = fmaf(gf[6], xf[6], s0);
              s1 = fmaf(gf[7], xf[7], s1);
              acc[u][i] += s0 + s1;
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int i = 0; i < n; ++i) {
            const float v = warp_sum(acc[u][i]);
            if (lane == tt + u) mine[i] = v;
          }
      }
      // (2) send my token's partial to its owner
      if (tid == 0) MHC_BWD_TRACE(1);
      const int pb = j % RB;
      const uint32_t pph = (j / RB) & 1;
      const int row = wp * 32 + lane;
      mbar_wait<true>(bar(B::p_free + pb), pph ^ 1, wc);
      {
        const int owner = row / TPO;
        const uint32_t dst = mapa_shared(smem_u32(pdh + (pb * kBM + (int)rank * TPO + (row % TPO)) * n), owner);
#pragma unroll
        for (int i = 0; i < n; ++i) st_cluster_f32(dst + 4 * i, mine[i]);
        mbar_arrive_remote(bar(B::p_full + pb), owner);
      }
      // (3) owner: reduce the C partials of my TPO tokens in rank order
      mbar_wait<true>(bar(B::p_full + pb), pph, wc);
      if (tid == 0) MHC_BWD_TRACE(2);
      for (int idx = tid; idx < TPO * n; idx += 128) {
        const int lt = idx / n, i = idx - lt * n;
        float s = 0.f;
        for (int src = 0; src < C; ++src) s += pdh[(pb * kBM + src * TPO + lt) * n + i];
        dhp_s[lt * n + i] = s;
      }
      named_sync(1, 128);
      if (tid < C) mbar_arrive_remote(bar(B::p_free + pb), tid);   // one release per destination CTA
      // one thread per owned token: dh_mix, c and the dalpha / dbias terms
      for (int lt = tid; lt < TPO; lt += 128) {
        const int64_t t = (int64_t)tile * kBM + (int)rank * TPO + lt;
        const bool valid = t < p.T;
        const float* oi = own_in + lt * Cf::OWNW;
        const float ir = oi[Cf::OWN_IN - 1];
        float dinv = 0.f, dal0 = 0.f, dal1 = 0.f, dal2 = 0.f;
#pragma unroll
        for (int jj = 0; jj < N_OUT; ++jj) {
          const float hm = oi[jj];
          float g2, tmp;
          if (jj < n) {
            const float s = oi[N_OUT + jj] - p.hc_eps;
            g2 = dhp_s[lt * n + jj] * s * (1.0f - s);
            tmp = a_pre * g2;
          } else if (jj < 2 * n) {
            const float hq = oi[N_OUT + n + (jj - n)];
            g2 = oi[N_OUT + 2 * n + (jj - n)] * hq * (1.0f - hq / 2.0f);
            tmp = a_post * g2;
          } else {
            g2 = oi[N_OUT + 3 * n + (jj - 2 * n)];
            tmp = a_res * g2;
          }
          if (!valid) g2 = tmp = 0.f;
          rec_s[lt * RECW + jj] = tmp * ir;                 // dh_mix (golden.py:62)
          dinv += tmp * hm;                                 // dinv_rms (golden.py:74)
          const float dal = g2 * (hm * ir);                 // dalpha terms (golden.py:77-79)
          if (jj < n) dal0 += dal;
          else if (jj < 2 * n) dal1 += dal;
          else dal2 += dal;
          contrib[lt * Cf::CW + 3 + jj] = g2;               // dbias terms (golden.py:83-85)
        }
        contrib[lt * Cf::CW + 0] = dal0;
        contrib[lt * Cf::CW + 1] = dal1;
        contrib[lt * Cf::CW + 2] = dal2;
        rec_s[lt * RECW + N_OUT] = valid ? dinv * (ir * ir * ir) * inv_nd : 0.f;   // c (golden.py:89)
#pragma unroll
        for (int i = 0; i < n; ++i) rec_s[lt * RECW + N_OUT + 1 + i] = valid ? oi[N_OUT + i] : 0.f;
        for (int w = N_OUT + 1 + n; w < RECW; ++w) rec_s[lt * RECW + w] = 0.f;
      }
      named_sync(1, 128);
      // running dalpha / dbias columns of this CTA's owned tokens, fixed order
      if (tid < Cf::CW)
        for (int lt = 0; lt < TPO; ++lt) ab_acc += contrib[lt * Cf::CW + tid];
      named_sync(1, 128);
      // (4) broadcast the records of my tokens to every CTA of the cluster
      mbar_wait<true>(bar(B::bc_free), (j & 1) ^ 1, wc);
      for (int idx = tid; idx < TPO * C; idx += 128) {
        const int lt = idx % TPO, dstc = idx / TPO;
        const uint32_t dst = mapa_shared(smem_u32(bc + ((int)rank * TPO + lt) * RECW), dstc);
#pragma unroll
        for (int w = 0; w < RECW; w += 4)
          st_cluster_v4_f32(dst + 4 * w, rec_s[lt * RECW + w], rec_s[lt * RECW + w + 1], rec_s[lt * RECW + w + 2],
                            rec_s[lt * RECW + w + 3]);
        mbar_arrive_remote(bar(B::bc_full), dstc);
      }
      named_sync(1, 128);
      if (tid == 0) MHC_BWD_TRACE(3);
    }
    if (tid < Cf::CW) p.abpart[((int64_t)cid * C + rank) * Cf::CW + tid] = ab_acc;
  } else {
    // ------------------------------------------------ WG_E: operands, dx epilogue, G flush
    // 8 warps: two per TMEM lane quadrant; eh selects the half of the columns.
    const int q4 = warp & 3;
    const int eh = (warp - kWarpE0) >> 2;
    const int row = 32 * q4 + lane;          // token row = TMEM lane
    const bool issuer = (q4 == 0 && lane == 0 && eh == 0);
    const uint64_t pol_out = l2_policy_evict_first();   // dx must not push out data awaiting re-read
    uint32_t q = 0, dq = 0, flushes = 0;
    for (int j = 0; j < my_tiles; ++j) {
      const int tile = (int)cid + j * (int)ncl;
      // (a) record -> DHM row of this token (the three bf16 terms of dh_mix)
      mbar_wait<true>(bar(B::bc_full), j & 1, wc);
      if (issuer) MHC_BWD_TRACE(4);
      mbar_wait(bar(B::dhm_free), (j & 1) ^ 1, wc);
      const float* rec = bc + row * RECW;
      const float c_t = rec[N_OUT];
      float hp[n];
#pragma unroll
      for (int i = 0; i < n; ++i) hp[i] = rec[N_OUT + 1 + i];
      // DHM row: segment e holds term e of dh_mix[0..N_OUT), zero padded to SEGW;
      // this half writes every other 16-byte chunk of the row.
#pragma unroll
      for (int kc0 = 0; kc0 < Cf::KA / 8; kc0 += 2) {
        const int kc = kc0 + eh;
        const int e = (kc * 8) / Cf::SEGW, j0 = kc * 8 - e * Cf::SEGW;
        uint32_t w[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          uint32_t lohi[2];
#pragma unroll
          for (int b2 = 0; b2 < 2; ++b2) {
            const int jj = j0 + h * 2 + b2;
            lohi[b2] = jj < N_OUT ? split_term(rec[jj], e) : 0;
          }
          w[h] = lohi[0] | (lohi[1] << 16);
        }
        *reinterpret_cast<uint4*>(dhm + interleave_off(row, kc * 8, Cf::RG_BYTES)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(bar(B::dhm_full));
      named_sync(2, kThreadsE);
      if (issuer) MHC_BWD_TRACE(5);
      if (q4 == 0 && eh == 0 && lane < C) mbar_arrive_remote(bar(B::bc_free), lane);
      // (b) dx of every 64-k block of the slice
      for (int dch = 0; dch < DCH; ++dch, ++dq) {
        const int ds = dq % Cf::DS;
        mbar_wait(bar(B::dh_full + ds), (dq / Cf::DS) & 1, wc);
        const uint32_t dh_row = smem_u32(dhr + ds * Cf::X_BYTES) + row * 128;
        for (int i = 0; i < n; ++i, ++q) {
          const int s = q % Cf::XS;
          const int dvb = DVB == 2 ? (int)(q & 1) : 0;
          const uint32_t dvph = DVB == 2 ? (q >> 1) & 1 : q & 1;
          mbar_wait(bar(B::x_full + s), (q / Cf::XS) & 1, wc);
          if (issuer) MHC_BWD_TRACE_Q(5);
          mbar_wait(bar(B::dv_full + dvb), dvph, wc);
          if (issuer) MHC_BWD_TRACE_Q(6);
          tc_fence_after();
          const uint32_t x_row = smem_u32(xr + s * Cf::X_BYTES) + row * 128;
          const uint32_t gm = smem_u32(gam_s + i * Dc + dch * kBK);
          float v[32];
          {
            float v0[16], v1[16];
            const uint32_t ta = tmem_dv + dvb * 64 + ((uint32_t)(32 * q4) << 16) + eh * 32;
            tmem_ld16(ta, v0);
            tmem_ld16(ta + 16, v1);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              v[e] = v0[e];
              v[16 + e] = v1[e];
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B::dv_empty + dvb));
          // the staging buffer is free once the previous TMA store has read it
          if (issuer) bulk_wait_read0();
          named_sync(2, kThreadsE);
          const uint32_t st_row = smem_u32(dxs) + row * 128;
#pragma unroll
          for (int hc = 0; hc < 4; ++hc) {
            const int c = eh * 4 + hc;                // 16-byte chunk 0..7 of the 128-byte row
            const uint32_t sw = (uint32_t)((c ^ (row & 7)) << 4);
            float xf[8], gf[8];
            bf16x8_to_f32(lds128(x_row + sw), xf);
            bf16x8_to_f32(lds128(dh_row + sw), gf);
            const uint4 ga = lds128(gm + c * 32), gb = lds128(gm + c * 32 + 16);
            const float gam[8] = {__uint_as_float(ga.x), __uint_as_float(ga.y), __uint_as_float(ga.z),
                                  __uint_as_float(ga.w), __uint_as_float(gb.x), __uint_as_float(gb.y),
                                  __uint_as_float(gb.z), __uint_as_float(gb.w)};
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              const float d0 = v[hc * 8 + e] * gam[e] + ((-c_t) * xf[e] + hp[i] * gf[e]);
              const float d1 = v[hc * 8 + e + 1] * gam[e + 1] + ((-c_t) * xf[e + 1] + hp[i] * gf[e + 1]);
              o[e / 2] = (uint32_t)f32_to_bf16_bits(d0) | ((uint32_t)f32_to_bf16_bits(d1) << 16);
            }
            sts128(st_row + sw, make_uint4(o[0], o[1], o[2], o[3]));
          }
          fence_proxy_async_smem();
          named_sync(2, kThreadsE);
          if (issuer && !*abort_flag) {
            tma_store_2d(&map_dx, smem_u32(dxs), i * D + (int)rank * Dc + dch * kBK, tile * kBM, pol_out);
            bulk_commit();
          }
          if (issuer) MHC_BWD_TRACE_Q(7);
          if (issuer && dch == 0 && i == 0) MHC_BWD_TRACE(6);
          if (issuer && dch == DCH - 1 && i == n - 1) MHC_BWD_TRACE(7);
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(bar(B::x_empty + s));
            if (i == n - 1) mbar_arrive(bar(B::dh_empty + ds));
          }
        }
      }
      // (c) flush G of the finished group into the per-cluster partial
      if ((j + 1) % p.FT == 0 || j == my_tiles - 1) {
        mbar_wait(bar(B::g_full), flushes & 1, wc);
        tc_fence_after();
        for (int blk = 0; blk < NPAIR; ++blk) {
          const int dch = blk / (n / 2), i0 = (blk % (n / 2)) * 2;
          const int i = i0 + (row >> 6);
          const int64_t k = (int64_t)i * D + (int64_t)rank * Dc + dch * kBK + (row & 63);
          float* gp = p.gpart + (int64_t)cid * N_OUT * nD + k;
          for (int c16 = eh; c16 < Cf::NG / 16; c16 += 2) {
            float v[16];
            tmem_ld16(tmem_g + blk * Cf::NG + ((uint32_t)(32 * q4) << 16) + c16 * 16, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int jj = c16 * 16 + e;
              if (jj < N_OUT) {
                if (flushes == 0) gp[(int64_t)jj * nD] = v[e];
                else red_add_f32(gp + (int64_t)jj * nD, v[e]);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B::g_empty));
        if (issuer) MHC_BWD_TRACE(8);
        ++flushes;
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  if (warp >= kWarpE0 && lane == 0 && (warp & 3) == 0 && ((warp - kWarpE0) >> 2) == 0)
    bulk_wait_all0();   // the dx stores this thread issued have completed
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  cluster_sync_all();
}

// phi [N_OUT, nD] f32 -> per 64-k block the K-major interleaved image W1
// reads as the B operand of dvecX: row kk, column e*SEGW + j holds bf16 term
// e (hi, mid, lo) of phi[j][block*64 + kk]; padding columns are zero.
template <int n>
__global__ void __launch_bounds__(256) phit_kernel(const float* __restrict__ phi, uint16_t* __restrict__ img,
                                                   int nD) {
  using Cf = Cfg<n>;
  const int64_t per_block = (int64_t)kBK * Cf::KA;
  const int64_t total = (int64_t)(nD / kBK) * per_block;
  for (int64_t idx = blockIdx.x * 256ll + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * 256) {
    const int64_t blk = idx / per_block;
    const int r = (int)(idx - blk * per_block);
    const int kk = r / Cf::KA, ca = r - kk * Cf::KA;
    const int e = ca / Cf::SEGW, jj = ca - e * Cf::SEGW;
    const uint16_t v = jj < Cf::N_OUT ? split_term(phi[(int64_t)jj * nD + blk * kBK + kk], e) : 0;
    img[blk * (Cf::PH_BYTES / 2) + interleave_off(kk, ca, Cf::RG_BYTES) / 2] = v;
  }
}

}  // namespace bwdtc
}  // namespace mhc
