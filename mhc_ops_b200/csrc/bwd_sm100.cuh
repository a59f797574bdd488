// Backward of the mHC pre-op on sm_100a, second half: tcgen05 GEMMs over
// per-token records.
//
// Math: src/backward/golden.py:38-96.  Per token t (row of x):
//   dh_pre[i] = sum_d dh_in[d] x[i,d]                                  (:51)
//   dh_mix    = [a_pre dh_pre2, a_post dh_post2, a_res dh_res] * inv_rms (:53-62)
//   c         = (sum_j dh_mix_tmp[j] h_mix[j]) inv_rms^3 / nD           (:74, :89)
//   dx[k]     = gamma[k] (dh_mix @ phi)[k] - c x[k] + h_pre[i] dh_in[d] (:65, :89-94)
// and over tokens: G = dh_mix^T x, dphi = G * gamma (:68-69), dgamma[k] =
// sum_j phi[j,k] G[j,k] (= sum_t x dvecX_mm, :93), dalpha (:77-80), dbias (:83-86).
//
// The whole-row reductions (dh_pre, c, dalpha, dbias) run first in a
// streaming kernel (rowdot.cuh, bwd_rows_kernel) that leaves one record per
// token {dh_mix, c, h_pre}.  This kernel does the rest.  CTA (s, g) owns the
// d-slice [s*Dc, (s+1)*Dc) of every stream and the 128-token tiles g, g+S_T,
// ... of the batch; CTAs never talk to each other.  When the tiles do not
// split evenly over the token groups and SMs are left over, the leftover
// tiles go to extra CTAs that each take whole d-slices of them (their own
// slot of the G partials), so the busiest CTA has the fewest tiles.  Per tile:
//   * W3 loads the tile's records (TMA, 16 KB); W0 streams the slice's x
//     blocks [128 tok x 64 k] and dh_in blocks (TMA, 128-B swizzle); W2 streams
//     the pre-laid-out split-phi images (3 bf16 terms of phi per k);
//   * WG_E turns the records into the UMMA operand DHM [128 tok x 3 segments]:
//     the 3 bf16 terms (hi, mid, lo) of dh_mix, each segment padded to a
//     multiple of 16 (double buffered: tile j+1's DHM is built during tile j);
//   * W1 issues tcgen05.mma per pair of stages (streams 2ip, 2ip+1 of a
//     64-k chunk): dvecX = dh_mix @ (phi * gamma) (gamma folded into the
//     split-phi images, so the epilogue has no gamma term) as one N=128
//     accumulation over the two stacked images, the sum over 6 (dh term, phi
//     term) products (smallest first: m.M, l.H, h.L, m.H, h.M, h.H; exact to
//     ~2^-23 in the fp32 sum), M=128 tok, K=segment; and the pair's G block,
//     x^T . DHM over the hi and mid terms as one N=64 accumulation (M=128 k,
//     K=128 tokens; x read MN-major straight from the two TMA stages, DHM
//     read MN-major).  Wide MMAs matter here: a tcgen05.mma costs ~45-65
//     cycles to issue whatever its N, so an N=128 MMA does twice the work of
//     an N=64 one for the same time;
//   * WG_E reads dvecX (TMEM lane = token) and writes dx through a TMA store
//     (two warp groups take alternate stages) and flushes each pair's G block
//     from TMEM into the token group's partial (first tile stores, later
//     tiles add; one thread per address, so the order is fixed).
#pragma once

#include "common.cuh"
#include "sm100.cuh"

#undef MHC_FILE_ID
#define MHC_FILE_ID 5   // debug-bounds site ids: 5 * 100000 + line

namespace mhc {
namespace bwdtc {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kWarpE0 = 4;          // first epilogue warp
constexpr int kThreadsE = 8 * 32;   // WG_E: 8 warps, two groups of one warp per TMEM lane quadrant
constexpr int kThreads = kWarpE0 * 32 + kThreadsE;   // W0, W1, W2, W3, WG_E(8)
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
  static constexpr int NG = SEGW;                        // G accumulator columns per 128-k block
  static constexpr int X_BYTES = kBM * 128;
  static constexpr int XS = 4;                           // x ring: two stage pairs
  static constexpr int DS = 1;                           // dh_in (held in registers for its n stages)
  static constexpr int PS = 4;                           // phi-image ring: two stage pairs
  static constexpr int RECW = round_up(N_OUT + 1 + n, 4);   // record: dh_mix, c, h_pre, pad
  static constexpr int REC_BYTES = kBM * RECW * 4;
  static constexpr int MAX_KC = 1024;                    // d-slice * n per CTA
  static constexpr int CW = 3 + N_OUT;                   // dalpha / dbias columns
  // tensor memory: G of a stage pair (hi and mid terms, 2 x SEGW columns) in
  // two buffers [0, 128), dvecX of a stage pair in two buffers [128, 384)
  static constexpr int G_BUF = 2 * SEGW;
  static constexpr int G_COLS = 2 * G_BUF;
  static constexpr int DV_COLS = 2 * kBK;

  static constexpr int smem_bytes() {
    return 1024 + XS * X_BYTES + DS * X_BYTES + PS * PH_BYTES + 2 * DHM_BYTES + 2 * X_BYTES /*dx staging*/ +
           REC_BYTES + 512;
  }
  static constexpr int SMEM = smem_bytes();
  static_assert(SMEM <= kSmemLimit, "backward tile does not fit in shared memory");
  static_assert(n % 2 == 0, "stages pair two streams of a d-chunk");
  static_assert(RECW == 32, "records are loaded as one 128-byte swizzled row per token");
  static_assert(G_COLS + 2 * DV_COLS <= 512, "TMEM budget");
  static_assert(G_BUF <= 256, "UMMA N of the G products");
};

struct Params {
  const uint8_t* phit;    // split images of phi * gamma, PH_BYTES per 64-k block
  float* gpart;           // [S_T][N_OUT][nD]
  int* status;
  int64_t T;
  int D;
  int Dc;                 // d-slice width (multiple of 64)
  int S_K;                // d-slices: D / Dc
  int S_T;                // token groups
  // leftover tiles (E > 0): main CTAs take J tiles each, E extra CTAs take
  // tiles 0 .. R-1 of ES whole d-slices each, into G-partial slot S_T
  int J;
  int E;
  int ES;
  int R;
  int num_tiles;
};

template <int n>
struct Bars {
  using Cf = Cfg<n>;
  static constexpr int x_full = 0;
  static constexpr int x_empty = x_full + Cf::XS;
  static constexpr int dh_full = x_empty + Cf::XS;
  static constexpr int dh_empty = dh_full + Cf::DS;
  static constexpr int ph_full = dh_empty + Cf::DS;      // per image pair
  static constexpr int ph_empty = ph_full + 2;
  static constexpr int dv_full = ph_empty + 2;           // per dvecX buffer (stage pair)
  static constexpr int dv_empty = dv_full + 2;
  static constexpr int dhm_full = dv_empty + 2;
  static constexpr int dhm_free = dhm_full + 2;
  static constexpr int g_full = dhm_free + 2;            // per G buffer
  static constexpr int g_empty = g_full + 2;
  static constexpr int rec_full = g_empty + 2;
  static constexpr int rec_free = rec_full + 1;
  static constexpr int count = rec_free + 1;
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
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  src = MHC_LDP(src, 16);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void red_add_f32(float* addr, float v) {
  addr = MHC_STP(addr, 4);
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

// One token's DHM row from its record: segment e holds bf16 term e of
// dh_mix[0..N_OUT), zero padded to SEGW (K-major interleaved image).  Half EH
// writes the 16-byte chunks kc = EH, EH+2, ... of the row; the partner warp
// of the other epilogue group writes the rest.
template <int n, int EH>
__device__ __forceinline__ void dhm_row_half(const float (&rec)[Cfg<n>::RECW], uint8_t* dst, int row) {
  using Cf = Cfg<n>;
#pragma unroll
  for (int kc = EH; kc < Cf::KA / 8; kc += 2) {
    const int e = (kc * 8) / Cf::SEGW, j0 = kc * 8 - e * Cf::SEGW;
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int ja = j0 + 2 * h, jb = ja + 1;
      const uint32_t lo = ja < Cf::N_OUT ? split_term(rec[ja < Cf::N_OUT ? ja : 0], e) : 0;
      const uint32_t hi = jb < Cf::N_OUT ? split_term(rec[jb < Cf::N_OUT ? jb : 0], e) : 0;
      w[h] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(dst + interleave_off(row, kc * 8, Cf::RG_BYTES)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <int n>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_kernel(const __grid_constant__ CUtensorMap map_x2d, const __grid_constant__ CUtensorMap map_dh,
               const __grid_constant__ CUtensorMap map_dx, const __grid_constant__ CUtensorMap map_rec,
               const Params p) {
  using Cf = Cfg<n>;
  using B = Bars<n>;
  constexpr int N_OUT = Cf::N_OUT;
  constexpr int RECW = Cf::RECW;
  constexpr int NP = n / 2;                              // stage pairs per d-chunk

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xr = smem;                                  // XS x blocks (pairs adjacent)
  uint8_t* dhr = xr + Cf::XS * Cf::X_BYTES;            // DS dh_in blocks
  uint8_t* phr = dhr + Cf::DS * Cf::X_BYTES;           // PS split-phi images (pairs adjacent)
  uint8_t* dhm = phr + Cf::PS * Cf::PH_BYTES;          // 2 x DHM: A of dvecX, B of G
  uint8_t* dxs = dhm + 2 * Cf::DHM_BYTES;              // 2 x dx staging [128 tok x 64] (128-B swizzle)
  float* recs = reinterpret_cast<float*>(dxs + 2 * Cf::X_BYTES);    // [128][RECW] records, 128-B swizzle
  uint64_t* bars = reinterpret_cast<uint64_t*>(recs + kBM * RECW);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B::count);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // This CTA's units (tile, d-slice), u = 0 .. my_tiles-1.  Main CTA (s, g):
  // d-slice s of tiles tiles-1-g, tiles-1-g-S_T, ... (last-first, so the first
  // ones re-read what the row kernel read last).  Extra CTA e: d-slices
  // e*ES .. e*ES+ES-1, each over the leftover tiles R-1 .. 0.
  const int nmain = p.S_K * p.S_T;
  const bool extra = (int)blockIdx.x >= nmain;
  const int slice0 = extra ? ((int)blockIdx.x - nmain) * p.ES : (int)blockIdx.x % p.S_K;
  const int group = extra ? p.S_T : (int)blockIdx.x / p.S_K;
  const int D = p.D;
  const int Dc = p.Dc;
  const int DCH = Dc / kBK;
  const int nD = n * D;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  auto tile_of = [&](int u) { return extra ? p.R - 1 - u % p.R : p.num_tiles - 1 - (group + u * p.S_T); };
  auto slice_of = [&](int u) { return extra ? slice0 + u / p.R : slice0; };
  // the unit opens this CTA's G partial of its d-slice: stored, not added
  auto first_of = [&](int u) { return extra ? u % p.R == 0 : u == 0; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < Cf::XS; ++i) {
      mbar_init(bar(B::x_full + i), 1);
      mbar_init(bar(B::x_empty + i), 1 + kThreadsE / 64);   // G commit + the stage's epilogue group
    }
    for (int i = 0; i < Cf::DS; ++i) {
      mbar_init(bar(B::dh_full + i), 1);
      mbar_init(bar(B::dh_empty + i), kThreadsE / 32);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B::ph_full + i), 32);   // one cp.async arrival per lane of W2
      mbar_init(bar(B::ph_empty + i), 1);
      mbar_init(bar(B::dv_full + i), 1);
      mbar_init(bar(B::dv_empty + i), kThreadsE / 32);    // both groups read their stage of the pair
      mbar_init(bar(B::dhm_full + i), kThreadsE);
      mbar_init(bar(B::dhm_free + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B::g_full + i), 1);
      mbar_init(bar(B::g_empty + i), kThreadsE / 64);   // the flushing epilogue group
    }
    mbar_init(bar(B::rec_full), 1);
    mbar_init(bar(B::rec_free), kThreadsE);
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
    prefetch_tensormap(&map_rec);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_g = tmem_base;                        // 2 x G_BUF: G of a stage pair
  const uint32_t tmem_dv = tmem_base + Cf::G_COLS;          // 2 x DV_COLS: dvecX of a stage pair
  const WaitCtx wc{abort_flag, p.status};
  const int my_tiles = extra ? p.ES * p.R
                             : p.E > 0 ? p.J : (group < p.num_tiles ? (p.num_tiles - 1 - group) / p.S_T + 1 : 0);
  const bool producer = (lane == 0);

  if (warp == 0) {
    // ------------------------------------------------ W0: TMA producer (x, dh_in)
    if (producer) {
      const uint64_t pol_drop = l2_policy_evict_first();
      uint32_t q = 0, dq = 0;
      for (int j = 0; j < my_tiles; ++j) {
        const int tile = tile_of(j);
        const int slice = slice_of(j);
        for (int dch = 0; dch < DCH; ++dch, ++dq) {
          const int ds = dq % Cf::DS;
          mbar_wait(bar(B::dh_empty + ds), ((dq / Cf::DS) & 1) ^ 1, wc);
          if (!*abort_flag) {
            mbar_arrive_expect_tx(bar(B::dh_full + ds), Cf::X_BYTES);
            tma_load_2d(smem_u32(dhr + ds * Cf::X_BYTES), &map_dh, bar(B::dh_full + ds), slice * Dc + dch * kBK,
                        tile * kBM, pol_drop);
          }
          for (int i = 0; i < n; ++i, ++q) {
            const int s = q % Cf::XS;
            const int k0 = i * D + slice * Dc + dch * kBK;
            mbar_wait(bar(B::x_empty + s), ((q / Cf::XS) & 1) ^ 1, wc);
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
    // Per stage pair (streams 2ip, 2ip+1 of a d-chunk): dvecX as one N=128
    // accumulation over the two stacked phi images, then G over the x pair.
    // Descriptors are built once and advanced by adding (bytes >> 4) to their
    // start-address field.
    if (producer) {
      constexpr uint32_t idesc_dv = idesc_bf16_f32(kBM, 2 * kBK, false, false);
      constexpr uint32_t idesc_g = idesc_bf16_f32(kBM, Cf::G_BUF, true, true);
      uint32_t pq = 0;
      for (int j = 0; j < my_tiles; ++j) {
        const int hb = j & 1;
        mbar_wait(bar(B::dhm_full + hb), (j >> 1) & 1, wc);
        tc_fence_after();
        const uint32_t dhm_a = smem_u32(dhm + hb * Cf::DHM_BYTES);
        const uint64_t a_dv = desc_kmajor_interleave(dhm_a, 128, Cf::RG_BYTES);      // DHM, K-major
        const uint64_t b_g = desc_kmajor_interleave(dhm_a, Cf::RG_BYTES, 128);       // DHM read MN-major
        for (int dch = 0; dch < DCH; ++dch) {
          for (int ip = 0; ip < NP; ++ip, ++pq) {
            const int pb = (int)(pq & 1);
            mbar_wait(bar(B::ph_full + pb), (pq >> 1) & 1, wc);
            mbar_wait(bar(B::dv_empty + pb), ((pq >> 1) & 1) ^ 1, wc);
            tc_fence_after();
            if (!*abort_flag) {
              const uint64_t b_dv = desc_kmajor_interleave(smem_u32(phr + pb * 2 * Cf::PH_BYTES), 128, Cf::RG_BYTES);
              const uint32_t d = tmem_dv + pb * Cf::DV_COLS;
#pragma unroll
              for (int pr = 0; pr < 6; ++pr) {
#pragma unroll
                for (int ks = 0; ks < Cf::SEGW / 16; ++ks) {
                  const uint32_t ca = (prod_a_term(pr) * Cf::SEGW + ks * 16) * 16;
                  const uint32_t cb = (prod_b_term(pr) * Cf::SEGW + ks * 16) * 16;
                  umma_bf16(d, a_dv + (ca >> 4), b_dv + (cb >> 4), idesc_dv, pr != 0 || ks != 0);
                }
              }
              umma_commit(bar(B::ph_empty + pb));
              umma_commit(bar(B::dv_full + pb));
            }
            // G over the x pair: rows 0..63 stream 2ip, 64..127 stream 2ip+1
            const uint32_t q0 = 2 * pq;
            const int s0 = (int)(q0 % Cf::XS);
            mbar_wait(bar(B::x_full + s0), (q0 / Cf::XS) & 1, wc);
            mbar_wait(bar(B::x_full + s0 + 1), ((q0 + 1) / Cf::XS) & 1, wc);
            mbar_wait(bar(B::g_empty + pb), ((pq >> 1) & 1) ^ 1, wc);
            tc_fence_after();
            if (!*abort_flag) {
              // N = the hi and mid segments of DHM (G needs ~2^-17), one N=64
              // accumulation over the tile's 128 tokens; flushed per pair
              const uint32_t d = tmem_g + pb * Cf::G_BUF;
              const uint64_t a_g = desc_mnmajor_sw128(smem_u32(xr + s0 * Cf::X_BYTES), Cf::X_BYTES, 1024);
#pragma unroll
              for (int ks = 0; ks < kBM / 16; ++ks)
                umma_bf16(d, a_g + ((ks * 2048) >> 4), b_g + ((ks * 2 * Cf::RG_BYTES) >> 4), idesc_g, ks != 0);
              umma_commit(bar(B::x_empty + s0));
              umma_commit(bar(B::x_empty + s0 + 1));
              umma_commit(bar(B::g_full + pb));
            }
          }
        }
        if (!*abort_flag) umma_commit(bar(B::dhm_free + hb));
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------ W2: split-phi image producer (one pair at a time)
    // The whole warp copies the two images with 16-byte cp.async (LSU path), so
    // the TMA engine only carries x, dh_in, the records and the dx stores.
    uint32_t pq = 0;
    for (int j = 0; j < my_tiles; ++j) {
      const int slice = slice_of(j);
      for (int dch = 0; dch < DCH; ++dch) {
        for (int ip = 0; ip < NP; ++ip, ++pq) {
          const int pb = (int)(pq & 1);
          mbar_wait(bar(B::ph_empty + pb), ((pq >> 1) & 1) ^ 1, wc);
          if (!*abort_flag) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int k0 = (2 * ip + h) * D + slice * Dc + dch * kBK;
              const uint8_t* src = p.phit + (size_t)(k0 / kBK) * Cf::PH_BYTES;
              const uint32_t dst = smem_u32(phr + (pb * 2 + h) * Cf::PH_BYTES);
#pragma unroll 4
              for (int off = lane * 16; off < Cf::PH_BYTES; off += 32 * 16) cp_async16(dst + off, src + off);
            }
          }
          cp_async_arrive_noinc(bar(B::ph_full + pb));   // fires when this lane's copies have landed
        }
      }
    }
  } else if (warp == 3) {
    // ------------------------------------------------ W3: record producer (one TMA box per tile)
    if (producer) {
      const uint64_t pol_keep = l2_policy_evict_last();   // every d-slice of the tile reads it
      for (int j = 0; j < my_tiles; ++j) {
        mbar_wait(bar(B::rec_free), (j & 1) ^ 1, wc);
        if (!*abort_flag) {
          mbar_arrive_expect_tx(bar(B::rec_full), Cf::REC_BYTES);
          tma_load_2d(smem_u32(recs), &map_rec, bar(B::rec_full), 0, tile_of(j) * kBM, pol_keep);
        }
      }
    }
  } else {
    // ------------------------------------------------ WG_E: operands, dx epilogue, G flush
    // 8 warps: two groups of four, one warp per TMEM lane quadrant each.  The
    // dx epilogue ping-pongs: group eh takes the stages q with q & 1 == eh
    // (columns eh*64.. of the pair's dvecX buffer, its own staging buffer),
    // so one group's TMEM -> smem -> TMA-store chain overlaps the other's.
    // For the DHM rows and the G flush eh selects the half of the columns.
    const int q4 = warp & 3;
    const int eh = (warp - kWarpE0) >> 2;
    const int row = 32 * q4 + lane;          // token row = TMEM lane
    const bool issuer = (q4 == 0 && lane == 0);   // one per group
    const uint64_t pol_out = l2_policy_evict_first();
    // Record of tile jj -> DHM buffer jj&1 (the three bf16 terms of dh_mix);
    // returns this row's c and h_pre.  Rows past the batch arrive zero-filled.
    auto build_dhm = [&](int jj, float& c_t, float (&hp)[n]) {
      mbar_wait(bar(B::rec_full), jj & 1, wc);
      mbar_wait(bar(B::dhm_free + (jj & 1)), ((jj >> 1) & 1) ^ 1, wc);
      // row `row` of the swizzled record box: 16-byte chunk c sits at c ^ (row & 7)
      float rec[RECW];
      {
        const uint32_t rb = smem_u32(recs) + row * 128;
#pragma unroll
        for (int c = 0; c < RECW / 4; ++c) {
          const uint4 v = lds128(rb + ((c ^ (row & 7)) << 4));
          rec[4 * c] = __uint_as_float(v.x);
          rec[4 * c + 1] = __uint_as_float(v.y);
          rec[4 * c + 2] = __uint_as_float(v.z);
          rec[4 * c + 3] = __uint_as_float(v.w);
        }
      }
      uint8_t* dst = dhm + (jj & 1) * Cf::DHM_BYTES;
      c_t = rec[N_OUT];
#pragma unroll
      for (int i = 0; i < n; ++i) hp[i] = rec[N_OUT + 1 + i];
      if (eh == 0) dhm_row_half<n, 0>(rec, dst, row);
      else dhm_row_half<n, 1>(rec, dst, row);
      fence_proxy_async_smem();
      mbar_arrive(bar(B::rec_free));
      mbar_arrive(bar(B::dhm_full + (jj & 1)));
    };
    float c_cur = 0.f, hp_cur[n];
    if (my_tiles > 0) build_dhm(0, c_cur, hp_cur);
    uint32_t q = 0, dq = 0;
    for (int j = 0; j < my_tiles; ++j) {
      const int tile = tile_of(j);
      const int slice = slice_of(j);
      const bool first = first_of(j);
      float c_nxt = 0.f, hp_nxt[n];
#pragma unroll
      for (int i = 0; i < n; ++i) hp_nxt[i] = 0.f;
      if (j + 1 < my_tiles) build_dhm(j + 1, c_nxt, hp_nxt);
      // dx of every 64-k block of the slice
      for (int dch = 0; dch < DCH; ++dch, ++dq) {
        const int ds = dq % Cf::DS;
        mbar_wait(bar(B::dh_full + ds), (dq / Cf::DS) & 1, wc);
        // this row's dh_in chunks serve the group's streams: read once, release
        uint4 dhv[8];
        {
          const uint32_t dh_row = smem_u32(dhr + ds * Cf::X_BYTES) + row * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) dhv[c] = lds128(dh_row + ((c ^ (row & 7)) << 4));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B::dh_empty + ds));
        for (int i = 0; i < n; ++i, ++q) {
          if ((int)(q & 1) != eh) continue;          // the other group's stage
          const int s = q % Cf::XS;
          const uint32_t pq = q >> 1;
          const int pb = (int)(pq & 1);
          mbar_wait(bar(B::x_full + s), (q / Cf::XS) & 1, wc);
          mbar_wait(bar(B::dv_full + pb), (pq >> 1) & 1, wc);
          tc_fence_after();
          const uint32_t x_row = smem_u32(xr + s * Cf::X_BYTES) + row * 128;
          const uint32_t st_buf = smem_u32(dxs) + eh * Cf::X_BYTES;
          const uint32_t st_row = st_buf + row * 128;
          float hpi = hp_cur[0];   // h_pre of stream i (selects keep hp_cur in registers)
#pragma unroll
          for (int k = 1; k < n; ++k)
            if (i == k) hpi = hp_cur[k];
          const float2 hp2 = make_float2(hpi, hpi), nc2 = make_float2(-c_cur, -c_cur);
          // this group's staging buffer is free once its previous store has read it
          if (issuer) bulk_wait_read0();
          named_sync(2 + eh, kThreadsE / 2);
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {           // 32 columns at a time
            float v[32];
            {
              float v0[16], v1[16];
              const uint32_t ta = tmem_dv + pb * Cf::DV_COLS + ((uint32_t)(32 * q4) << 16) + eh * kBK + hf * 32;
              tmem_ld16(ta, v0);
              tmem_ld16(ta + 16, v1);
              uint4 xv[4];
#pragma unroll
              for (int hc = 0; hc < 4; ++hc) xv[hc] = lds128(x_row + (((hf * 4 + hc) ^ (row & 7)) << 4));
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                v[e] = v0[e];
                v[16 + e] = v1[e];
              }
#pragma unroll
              for (int hc = 0; hc < 4; ++hc) {
                const int c = hf * 4 + hc;             // 16-byte chunk 0..7 of the 128-byte row
                float xf[8], gf[8];
                bf16x8_to_f32(xv[hc], xf);
                bf16x8_to_f32(dhv[c], gf);
                uint32_t o[4];
                // dx = (dvecX + h_pre dh_in) - c x, two elements per packed FMA
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                  float2 d = __ffma2_rn(hp2, make_float2(gf[e], gf[e + 1]),
                                        make_float2(v[hc * 8 + e], v[hc * 8 + e + 1]));
                  d = __ffma2_rn(nc2, make_float2(xf[e], xf[e + 1]), d);
                  o[e / 2] = pack_bf16x2(d.x, d.y);
                }
                sts128(st_row + (uint32_t)((c ^ (row & 7)) << 4), make_uint4(o[0], o[1], o[2], o[3]));
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B::dv_empty + pb));
          fence_proxy_async_smem();
          named_sync(2 + eh, kThreadsE / 2);
          if (issuer && !*abort_flag) {
            tma_store_2d(&map_dx, st_buf, i * D + slice * Dc + dch * kBK, tile * kBM, pol_out);
            bulk_commit();
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B::x_empty + s));
          if (pb == eh) {
            // G of this stage pair -> the token group's partial (rows 0..63
            // stream i & ~1, 64..127 the next); the same thread owns each
            // address in every tile: first tile stores, later tiles add
            mbar_wait(bar(B::g_full + pb), (pq >> 1) & 1, wc);
            tc_fence_after();
            const int ig = (i & ~1) + (row >> 6);
            float* gp = p.gpart + (int64_t)group * N_OUT * nD + (int64_t)ig * D + (int64_t)slice * Dc + dch * kBK +
                        (row & 63);
            const uint32_t tg = tmem_g + pb * Cf::G_BUF + ((uint32_t)(32 * q4) << 16);
#pragma unroll
            for (int c16 = 0; c16 < Cf::SEGW / 16; ++c16) {
              float hi[16], mid[16];
              tmem_ld16(tg + c16 * 16, hi);
              tmem_ld16(tg + Cf::SEGW + c16 * 16, mid);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const int jj = c16 * 16 + e;
                if (jj < N_OUT) {
                  const float v = mid[e] + hi[e];
                  if (first) MHC_ST(gp + (int64_t)jj * nD, v);
                  else red_add_f32(gp + (int64_t)jj * nD, v);
                }
              }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B::g_empty + pb));
          }
        }
      }
      c_cur = c_nxt;
#pragma unroll
      for (int i = 0; i < n; ++i) hp_cur[i] = hp_nxt[i];
    }
  }

  // ---------------------------------------------------------------- teardown
  if (warp >= kWarpE0 && lane == 0 && (warp & 3) == 0)
    bulk_wait_all0();   // the dx stores this thread (one issuer per epilogue group) issued have completed
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace bwdtc
}  // namespace mhc
