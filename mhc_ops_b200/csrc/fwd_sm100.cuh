// Forward of the mHC pre-op on sm_100a, first half: tcgen05 projection.
//
// Math: src/forward/golden.py:34-69 (h_mix = x @ phi^T pre-RMS, inv_rms,
// gates, h_in = sum_i h_pre[i] * x[i,:]).
//
// proj_kernel reads x once and leaves per token and K-slice the partial
// projection (pre-RMS h_mix) and the partial sum of x^2; the row half
// (rowdot.cuh, fwd_row_token) sums the partials in a fixed order, forms
// inv_rms and the gates and reads x a second time for h_in.  The partial rows
// of token t are parked in row t of h_in, which the row half reads before it
// overwrites that row with the result.  Two forms:
//   * fused (proj_kernel<n, true>, cooperative launch): extra warps WG_R run
//     the row half of every tile whose S_K units are all done (a counter per
//     tile in global memory, release/acquire), about one round of units
//     behind the projection, so the second read of x hits L2 (W0 loads x
//     with an evict-last hint);
//   * two kernels (proj_kernel<n, false> then rowdot::fwd_rows_kernel), for
//     shapes whose h_in row cannot hold the fused form's finer K-slices.
//
// Work units are (128-token tile, K-slice of KB_PER 64-wide K-blocks); a
// persistent grid walks them (in the two-kernel form with no communication
// between CTAs).  Per unit:
//   * W0 streams x (128 x 64 bf16, 128-B swizzle) and the bf16-split phi
//     block (NB x 64) of each K-block into an S-stage ring with TMA;
//   * W1 issues tcgen05.mma (M=128 tokens, N=NB split-phi rows, K=16); every
//     group of kKG K-blocks starts a fresh accumulator in a ring of NBUF TMEM
//     buffers;
//   * WG_F (4 warps, one thread per token row = TMEM lane) folds each group's
//     accumulator (all split terms) into its fp32 partials with
//     round-to-nearest adds -- the tensor core's own accumulation across many
//     K steps drifts (about 2^-23 per step, one-signed), across 8 it does not
//     -- and stores the unit's partial row (h_mix and WG_S's sum x^2, whole
//     32-byte sectors);
//   * WG_S (4 warps, one thread per token row; 2 warps with two rows a
//     thread in the fused bf16 form) sums x^2 of its rows from the
//     smem stages (tree per stage) and hands it to WG_F through shared memory.
// phi is split into NT bf16 terms (hi, mid[, lo]) stacked as UMMA N rows, so
// x (exact in bf16) times phi is exact to ~2^-(8*NT) before fp32 accumulation.
// Three terms at n <= 5: h_in's bound (one ulp plus 2^-18 of its terms) needs
// the gates to ~2^-18, which two terms miss when |h_mix| is large.
#pragma once

#include <cuda_fp8.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "rowdot.cuh"
#include "sm100.cuh"

#undef MHC_FILE_ID
#define MHC_FILE_ID 6   // debug-bounds site ids: 6 * 100000 + line

namespace mhc {
namespace fwdtc {

using namespace sm100;

constexpr int kBM = 128;          // tokens per tile = UMMA M = TMEM lanes
constexpr int kBK = 64;           // bf16 elements per 128-byte row
constexpr int kThreads = 10 * 32; // W0, W1, WG_F(4), WG_S(4)
constexpr int kRowWarps = 8;      // WG_R of the fused forward
// WG_S warps: 4 (a token row per thread), or 2 in the fused bf16 forward (two
// rows per thread), which leaves a 512-thread CTA and so up to 128 registers
// a thread, enough for the row warps to keep 6 chunks per lane in flight.
constexpr int s_warps(bool fused, bool fp8) { return fused && !fp8 ? 2 : 4; }
constexpr int threads_of(bool fused, bool fp8) { return (6 + s_warps(fused, fp8) + (fused ? kRowWarps : 0)) * 32; }
// 256-element chunks in flight per lane in the fused form's row warps (0:
// the row kernel's default).  Measured at the LLM shape with 128 registers a
// thread: 2, 3, 4, 5, 6 chunks gave a forward of 0.230, 0.223, 0.221, 0.229,
// 0.253 ms -- more loads in flight than 4 per lane slow the projection's
// stream more than they speed the row warps.
constexpr int fused_row_chunks(int n, bool fp8) { return !fp8 && n <= 4 ? 4 : 0; }
constexpr int kUnitSignals = 4;   // WG_F warps: arrivals on a tile's counter per unit
// Fused form: W0 starts this CTA's unit j only once WG_R has finished unit
// j - kRowLag.  Without a bound the projection can run away from the row
// warps, whose second read of x then misses L2 and slows them further.  The
// rows of a unit need only units of the same or the next round (a tile's
// S_K units are consecutive), so any kRowLag >= 2 cannot deadlock.
constexpr int kRowLag = 4;
constexpr int kKG = 2;            // K-blocks accumulated per TMEM accumulator
constexpr int kSmemLimit = 232448;

constexpr int round_up(int v, int a) { return (v + a - 1) / a * a; }
constexpr int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p *= 2;
  return p;
}

// Split terms of an fp32 phi: three at n <= 5, two above (see the top of
// this file).  A phi given in bf16 is exact in one term.
constexpr int default_terms(int n) { return n <= 5 ? 3 : 2; }

// kFp8: x comes as e4m3 bytes with a power-of-two scale per token; each
// stage also holds the raw fp8 box, which the sum-of-squares warps widen
// into the bf16 operand tile (exactly: every e4m3 value times a power of two
// is a bf16 value).
template <int n, int kNT = default_terms(n), bool kFp8 = false>
struct Cfg {
  static constexpr int N_OUT = n * n + 2 * n;
  static constexpr int NT = kNT;                           // phi split terms
  static constexpr int NB = round_up(NT * N_OUT, 16);      // UMMA N
  static constexpr int RW = round_up(N_OUT + 1, 8);        // floats per partial row (whole 32-byte sectors)
  static constexpr int A_BYTES = kBM * 128;
  static constexpr int B_BYTES = NB * 128;
  static constexpr int RAW_BYTES = kFp8 ? kBM * kBK : 0;   // fp8 box [128 tok x 64 k], after A and B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + RAW_BYTES;
  static constexpr int ACC_COLS = round_up(NB, 32);
  static constexpr int NBUF = (512 / ACC_COLS) < 4 ? (512 / ACC_COLS) : 4;   // accumulator ring
  static constexpr int TMEM_COLS = pow2_at_least(NBUF * ACC_COLS);
  static constexpr int SQ_BYTES = 2 * kBM * 4;              // WG_S -> WG_F hand-over of sum x^2, two units
  static constexpr int smem_bytes(int S) {
    return 1024 /*align slack*/ + S * STAGE_BYTES + SQ_BYTES + 512 /*barriers*/;
  }
  static constexpr int pick_stages() {
    int s = 8;
    while (s > 2 && smem_bytes(s) > kSmemLimit) --s;
    return s;
  }
  static constexpr int S = pick_stages();
  static constexpr int SMEM = smem_bytes(S);
  static_assert(SMEM <= kSmemLimit, "forward stage ring does not fit in shared memory");
  static_assert(STAGE_BYTES % 1024 == 0, "stages keep the 128-B swizzle atoms aligned");
  static_assert(RW % 4 == 0, "partial rows are stored as float4");
  static_assert(NB <= 256, "UMMA N above 256");
  static_assert(NBUF >= 2 && TMEM_COLS <= 512, "TMEM accumulator ring");
};

struct Params {
  float* part;            // partial rows: unit (tile, ks), token t -> part + t * part_stride + ks * RW
  int64_t part_stride;    // floats between consecutive tokens' partial areas (row pitch of h_in / 2)
  int* status;
  int64_t T;
  int S_K;                // K-slices
  int KB_PER;             // K-blocks per slice
  int num_units;          // tiles * S_K
  // fused forward only
  int* tile_done;         // [tiles] zeroed before the launch; kUnitSignals arrivals per finished unit
  rowdot::FwdRowArgs rows;
};

template <int n, int kNT, bool kFp8>
struct Bars {
  using Cf = Cfg<n, kNT, kFp8>;
  static constexpr int full = 0;
  static constexpr int empty = full + Cf::S;
  static constexpr int conv = empty + Cf::S;               // fp8: the stage's bf16 tile is written
  static constexpr int acc_full = conv + Cf::S;
  static constexpr int acc_empty = acc_full + Cf::NBUF;
  static constexpr int sq_full = acc_empty + Cf::NBUF;   // 2: WG_S wrote a unit's sum x^2
  static constexpr int sq_empty = sq_full + 2;           // 2: WG_F read it
  static constexpr int count = sq_empty + 2;
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

// One warp's arrival on its tile's counter after its partial stores: every
// lane fences its own stores, then lane 0 adds with release semantics.
__device__ __forceinline__ void signal_unit(int* counter, int lane) {
  __threadfence();
  __syncwarp();
  if (lane == 0) red_release_add(counter, 1);
}

// W0 of the fused form: wait until every WG_R warp has finished `need` units
// (a progress hint in shared memory, no data passes); bounded like mbar_wait.
__device__ __forceinline__ void wait_rows_done(volatile int* rows_done, int need, const WaitCtx& w) {
  uint64_t t0 = 0;
  for (uint32_t spin = 0;; ++spin) {
    int m = rows_done[0];
#pragma unroll
    for (int i = 1; i < kRowWarps; ++i) m = min(m, rows_done[i]);
    if (m >= need || *w.abort) return;
    __nanosleep(128);
    if ((spin & 255) == 0) {
      const uint64_t now = globaltimer_ns();
      if (spin == 0) {
        t0 = now;
      } else if (now - t0 > kWaitTimeoutNs) {
        *w.abort = 1;
        set_device_status(w.status, MHC_ERR_DEVICE_TIMEOUT);
        return;
      }
    }
  }
}

// Adds the accumulator columns of outputs [J0, J0 + JN) into part[0 .. JN):
// column t*N_OUT + j holds term t of output j; the terms of an output are
// summed smallest first, then added to its running partial (the same order
// as the one-group fold below, so both give the same bits).
template <int N_OUT, int NT, int J0, int JN>
__device__ __forceinline__ void fold_outputs(uint32_t taddr, float (&part)[JN]) {
  static_assert(J0 % 16 == 0 && JN % 16 == 0, "whole 16-column loads");
#pragma unroll
  for (int c16 = 0; c16 < JN / 16; ++c16) {
    float w[NT][16];
#pragma unroll
    for (int t = 0; t < NT; ++t) tmem_ld16(taddr + t * N_OUT + J0 + c16 * 16, w[t]);
    tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      float v = w[NT - 1][e];
#pragma unroll
      for (int tt = NT - 2; tt >= 0; --tt) v += w[tt][e];
      part[c16 * 16 + e] += v;
    }
  }
}

template <int n, bool kFused, int kNT = default_terms(n), bool kFp8 = false>
__global__ void __launch_bounds__(threads_of(kFused, kFp8), 1)
    proj_kernel(const __grid_constant__ CUtensorMap map_x2d, const __grid_constant__ CUtensorMap map_phi,
                const Params p) {
  using Cf = Cfg<n, kNT, kFp8>;
  using B = Bars<n, kNT, kFp8>;
  constexpr int N_OUT = Cf::N_OUT;
  constexpr int S = Cf::S;
  constexpr int SW = s_warps(kFused, kFp8);   // WG_S warps
  constexpr int RPT = 4 / SW;                 // token rows per WG_S thread
  constexpr int kRow0 = 6 + SW;               // first WG_R warp
  // n = 8 (80 outputs), bf16 x: the fold is split over two warp groups so
  // that no thread holds all 80 partials (which spilled): WG_F outputs
  // [0, 48), WG_S outputs [48, 80) and the sum of x^2, each storing its part
  // of the row.  Not for fp8 x, whose WG_S also widens every stage.
  constexpr bool kSplit = (N_OUT == 80) && !kFp8;
  constexpr int JF = kSplit ? 48 : N_OUT;   // outputs WG_F folds
  static_assert(!(kSplit && kFused), "the fused form signals a unit from WG_F alone");
  static_assert(!kSplit || SW == 4, "the split fold reads TMEM with all four WG_S lane quadrants");
  static_assert(!kSplit || (Cf::RW == 88 && JF % 4 == 0), "partial-row halves on 16-byte boundaries");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sq_buf = reinterpret_cast<float*>(ring + S * Cf::STAGE_BYTES);   // [2][kBM]
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + S * Cf::STAGE_BYTES + Cf::SQ_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B::count);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* rows_done = reinterpret_cast<volatile int*>(tmem_slot + 2);   // fused: [kRowWarps] units done

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto bar = [&](int i) { return smem_u32(&bars[i]); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(bar(B::full + i), 1);
      mbar_init(bar(B::empty + i), 1 + SW);   // MMA commit + the WG_S warps
      mbar_init(bar(B::conv + i), SW);        // fp8: the WG_S warps wrote the bf16 tile
    }
    for (int i = 0; i < Cf::NBUF; ++i) {
      mbar_init(bar(B::acc_full + i), 1);
      mbar_init(bar(B::acc_empty + i), kSplit ? 8 : 4);   // the folding warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B::sq_full + i), SW);
      mbar_init(bar(B::sq_empty + i), 4);
    }
    *abort_flag = 0;
    if (kFused)
      for (int i = 0; i < kRowWarps; ++i) rows_done[i] = 0;
    fence_mbarrier_init_cluster();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cf::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&map_x2d);
    prefetch_tensormap(&map_phi);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtx wc{abort_flag, p.status};
  const int KB = p.KB_PER;

  if (warp == 0) {
    // ------------------------------------------------ W0: TMA producer
    if (lane == 0) {
      // fused: x stays in L2 for WG_R's second read of the same rows
      const uint64_t pol_x = kFused ? l2_policy_evict_last() : l2_policy_evict_first();
      const uint64_t pol_phi = l2_policy_evict_last();
      uint32_t it = 0;
      int lu = 0;   // this CTA's unit count
      for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++lu) {
        const int tile = u / p.S_K, ks = u - (u / p.S_K) * p.S_K;
        if constexpr (kFused) {
          if (lu >= kRowLag) wait_rows_done(rows_done, lu - kRowLag + 1, wc);
        }
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          const int k0 = (ks * KB + kb) * kBK;
          mbar_wait(bar(B::empty + s), ((it / S) & 1) ^ 1, wc);
          if (*abort_flag) continue;
          uint8_t* st = ring + s * Cf::STAGE_BYTES;
          if constexpr (kFp8) {
            mbar_arrive_expect_tx(bar(B::full + s), Cf::B_BYTES + Cf::RAW_BYTES);
            tma_load_2d(smem_u32(st + Cf::A_BYTES + Cf::B_BYTES), &map_x2d, bar(B::full + s), k0, tile * kBM, pol_x);
          } else {
            mbar_arrive_expect_tx(bar(B::full + s), Cf::STAGE_BYTES);
            tma_load_2d(smem_u32(st), &map_x2d, bar(B::full + s), k0, tile * kBM, pol_x);
          }
          tma_load_2d(smem_u32(st + Cf::A_BYTES), &map_phi, bar(B::full + s), k0, 0, pol_phi);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ W1: tcgen05.mma issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kBM, Cf::NB, false, false);
      uint32_t it = 0, g = 0;
      for (int u = blockIdx.x; u < p.num_units; u += gridDim.x) {
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          const int ab = g % Cf::NBUF;
          const bool first = (kb % kKG) == 0, last = (kb % kKG) == kKG - 1 || kb == KB - 1;
          mbar_wait(bar((kFp8 ? B::conv : B::full) + s), (it / S) & 1, wc);
          if (first) mbar_wait(bar(B::acc_empty + ab), ((g / Cf::NBUF) & 1) ^ 1, wc);
          tc_fence_after();
          if (!*abort_flag) {
            const uint8_t* st = ring + s * Cf::STAGE_BYTES;
            const uint64_t a0 = desc_kmajor_sw128(smem_u32(st));
            const uint64_t b0 = desc_kmajor_sw128(smem_u32(st + Cf::A_BYTES));
            const uint32_t d_tmem = tmem_base + ab * Cf::ACC_COLS;
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) umma_bf16(d_tmem, a0 + 2 * kk, b0 + 2 * kk, idesc, !first || kk != 0);
            umma_commit(bar(B::empty + s));
            if (last) umma_commit(bar(B::acc_full + ab));
          }
          if (last) ++g;
        }
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------ WG_F: fold accumulators, store partial h_mix
    const int q = warp & 3;                   // TMEM lane quadrant of this warp
    const int row = 32 * q + lane;            // token row of the tile = TMEM lane
    uint32_t g = 0, uc = 0;
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++uc) {
      const int tile = u / p.S_K, ks = u - (u / p.S_K) * p.S_K;
      if constexpr (kSplit) {
        float part[JF];
#pragma unroll
        for (int jj = 0; jj < JF; ++jj) part[jj] = 0.f;
        for (int kb = 0; kb < KB; kb += kKG, ++g) {
          const int ab = g % Cf::NBUF;
          mbar_wait(bar(B::acc_full + ab), (g / Cf::NBUF) & 1, wc);
          tc_fence_after();
          fold_outputs<N_OUT, Cf::NT, 0, JF>(tmem_base + ((uint32_t)(32 * q) << 16) + ab * Cf::ACC_COLS, part);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B::acc_empty + ab));
        }
        const int64_t t = (int64_t)tile * kBM + row;
        if (t < p.T && !*abort_flag) {
          float4* dst = reinterpret_cast<float4*>(p.part + t * p.part_stride + (int64_t)ks * Cf::RW);
#pragma unroll
          for (int c = 0; c < JF / 4; ++c)
            MHC_ST(dst + c, make_float4(part[4 * c], part[4 * c + 1], part[4 * c + 2], part[4 * c + 3]));
        }
      } else {
      float part[N_OUT];
#pragma unroll
      for (int jj = 0; jj < N_OUT; ++jj) part[jj] = 0.f;
      for (int kb = 0; kb < KB; kb += kKG, ++g) {
        const int ab = g % Cf::NBUF;
        // column t*N_OUT + j of the accumulator holds term t of output j
        mbar_wait(bar(B::acc_full + ab), (g / Cf::NBUF) & 1, wc);
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + ab * Cf::ACC_COLS;
        if constexpr (N_OUT % 16 == 0 && Cf::NT == 2) {
          // wide outputs: 16 outputs at a time, both terms (mid + hi) before the add
#pragma unroll
          for (int c16 = 0; c16 < N_OUT / 16; ++c16) {
            float hi[16], mid[16];
            tmem_ld16(taddr + c16 * 16, hi);
            tmem_ld16(taddr + N_OUT + c16 * 16, mid);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) part[c16 * 16 + e] += mid[e] + hi[e];
          }
        } else {
          float v[Cf::NB];
#pragma unroll
          for (int c16 = 0; c16 < Cf::NB / 16; ++c16) {
            float w[16];
            tmem_ld16(taddr + c16 * 16, w);
#pragma unroll
            for (int e = 0; e < 16; ++e) v[c16 * 16 + e] = w[e];
          }
          tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < N_OUT; ++jj) {
            float t3 = v[(Cf::NT - 1) * N_OUT + jj];     // smallest term first
#pragma unroll
            for (int tt = Cf::NT - 2; tt >= 0; --tt) t3 += v[tt * N_OUT + jj];
            part[jj] += t3;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B::acc_empty + ab));
      }
      // this row's sum x^2 from WG_S, then the whole partial row (every
      // 32-byte sector written in full) with 16-byte stores
      const int sb = (int)(uc & 1);
      mbar_wait(bar(B::sq_full + sb), (uc >> 1) & 1, wc);
      const float sq = sq_buf[sb * kBM + row];
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B::sq_empty + sb));
      const int64_t t = (int64_t)tile * kBM + row;
      if (t < p.T && !*abort_flag) {
        float rowv[Cf::RW];
#pragma unroll
        for (int jj = 0; jj < Cf::RW; ++jj) rowv[jj] = jj < N_OUT ? part[jj < N_OUT ? jj : 0] : (jj == N_OUT ? sq : 0.f);
        float4* dst = reinterpret_cast<float4*>(p.part + t * p.part_stride + (int64_t)ks * Cf::RW);
#pragma unroll
        for (int c = 0; c < Cf::RW / 4; ++c)
          MHC_ST(dst + c, make_float4(rowv[4 * c], rowv[4 * c + 1], rowv[4 * c + 2], rowv[4 * c + 3]));
      }
      if constexpr (kFused) signal_unit(p.tile_done + tile, lane);
      }
    }
  } else if (warp < 6 + SW && RPT == 2) {
    // ------------------------------------------------ WG_S (fused bf16 form, 2 warps): sum of squares
    // Thread (w, lane) sums x^2 of token rows 32 w + lane and 32 (w + 2) + lane
    // of each stage, in the same order as the one-row-per-thread form below.
    const int w = warp - 6;
    uint32_t it = 0, uc = 0;
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++uc) {
      float sq[2] = {0.f, 0.f};
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S;
        mbar_wait(bar(B::full + s), (it / S) & 1, wc);
        uint4 xv[2][8];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int row = 32 * (w + 2 * r) + lane;
          const uint32_t base = smem_u32(ring + s * Cf::STAGE_BYTES) + row * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) xv[r][c] = lds128(base + (((c + row) & 7) << 4));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B::empty + s));
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          float c8[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float f[8];
            bf16x8_to_f32(xv[r][c], f);
            const float a = fmaf(f[0], f[0], f[1] * f[1]) + fmaf(f[2], f[2], f[3] * f[3]);
            const float b = fmaf(f[4], f[4], f[5] * f[5]) + fmaf(f[6], f[6], f[7] * f[7]);
            c8[c] = a + b;
          }
          sq[r] += ((c8[0] + c8[1]) + (c8[2] + c8[3])) + ((c8[4] + c8[5]) + (c8[6] + c8[7]));
        }
      }
      const int sb = (int)(uc & 1);
      mbar_wait(bar(B::sq_empty + sb), ((uc >> 1) & 1) ^ 1, wc);
      sq_buf[sb * kBM + 32 * w + lane] = sq[0];
      sq_buf[sb * kBM + 32 * (w + 2) + lane] = sq[1];
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B::sq_full + sb));
    }
  } else if (warp < 6 + SW) {
    // ------------------------------------------------ WG_S: sum of squares, store partial sum x^2
    const int row = 32 * (warp & 3) + lane;   // token row of the tile = smem row
    uint32_t it = 0, uc = 0, g = 0;
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++uc) {
      float sq = 0.f;
      constexpr int JS = kSplit ? N_OUT - JF : 16;   // outputs WG_S folds (n = 8)
      float part[JS];
#pragma unroll
      for (int jj = 0; jj < JS; ++jj) part[jj] = 0.f;
      float scale = 1.f;   // fp8: 2^e of this row's token (rows past the batch are zero anyway)
      if constexpr (kFp8) {
        const int64_t t = (int64_t)(u / p.S_K) * kBM + row;
        if (p.rows.x_exp != nullptr && t < p.T) scale = ldexpf(1.0f, (int)MHC_LDG(p.rows.x_exp + t));
      }
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S;
        mbar_wait(bar(B::full + s), (it / S) & 1, wc);
        const uint32_t base = smem_u32(ring + s * Cf::STAGE_BYTES) + row * 128;
        uint4 xv[8];
        if constexpr (kFp8) {
          // widen the row's 64 e4m3 values into the bf16 tile, 128-B swizzled
          // as a TMA load would have written it (16-byte chunk c of row r at
          // chunk c ^ (r & 7)), then read the row back in the bf16 path's
          // order, so the sum of squares adds the same values in the same order
          const uint32_t raw = smem_u32(ring + s * Cf::STAGE_BYTES + Cf::A_BYTES + Cf::B_BYTES) + row * kBK;
          uint4 lx[8];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const uint4 r = lds128(raw + h * 16);
            const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
              uint32_t o[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint32_t pair = w[2 * c2 + q / 2] >> (16 * (q & 1));
                const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(pair & 0xFFFFu), __NV_E4M3);
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
                o[q] = pack_bf16x2(f.x * scale, f.y * scale);
              }
              lx[2 * h + c2] = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
#pragma unroll
          for (int c = 0; c < 8; ++c) sts128(base + ((c ^ (row & 7)) << 4), lx[c]);
#pragma unroll
          for (int c = 0; c < 8; ++c) xv[c] = lds128(base + (((c + row) & 7) << 4));   // the bf16 path's order
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(bar(B::conv + s));
            mbar_arrive(bar(B::empty + s));
          }
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) xv[c] = lds128(base + (((c + row) & 7) << 4));
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(B::empty + s));
        }
        float c8[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float f[8];
          bf16x8_to_f32(xv[c], f);
          const float a = fmaf(f[0], f[0], f[1] * f[1]) + fmaf(f[2], f[2], f[3] * f[3]);
          const float b = fmaf(f[4], f[4], f[5] * f[5]) + fmaf(f[6], f[6], f[7] * f[7]);
          c8[c] = a + b;
        }
        sq += ((c8[0] + c8[1]) + (c8[2] + c8[3])) + ((c8[4] + c8[5]) + (c8[6] + c8[7]));
        if constexpr (kSplit) {
          if ((kb % kKG) == kKG - 1 || kb == KB - 1) {   // the accumulator of this K-block group is complete
            const int ab = g % Cf::NBUF;
            mbar_wait(bar(B::acc_full + ab), (g / Cf::NBUF) & 1, wc);
            tc_fence_after();
            fold_outputs<N_OUT, Cf::NT, JF, JS>(tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) + ab * Cf::ACC_COLS,
                                                 part);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B::acc_empty + ab));
            ++g;
          }
        }
      }
      if constexpr (kSplit) {
        // outputs [48, 80), sum x^2 and the zero padding of the partial row
        const int64_t t = (int64_t)(u / p.S_K) * kBM + row;
        const int ks = u - (u / p.S_K) * p.S_K;
        if (t < p.T && !*abort_flag) {
          float rowv[Cf::RW - JF];
#pragma unroll
          for (int jj = 0; jj < Cf::RW - JF; ++jj) rowv[jj] = jj < JS ? part[jj < JS ? jj : 0] : (jj == JS ? sq : 0.f);
          float4* dst = reinterpret_cast<float4*>(p.part + t * p.part_stride + (int64_t)ks * Cf::RW + JF);
#pragma unroll
          for (int c = 0; c < (Cf::RW - JF) / 4; ++c)
            MHC_ST(dst + c, make_float4(rowv[4 * c], rowv[4 * c + 1], rowv[4 * c + 2], rowv[4 * c + 3]));
        }
        continue;
      }
      // hand the unit's sum x^2 to WG_F, which stores the partial row
      const int sb = (int)(uc & 1);
      mbar_wait(bar(B::sq_empty + sb), ((uc >> 1) & 1) ^ 1, wc);
      sq_buf[sb * kBM + row] = sq;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B::sq_full + sb));
    }
  } else {
    if constexpr (kFused) {
      // ---------------------------------------------- WG_R: gates, outputs and h_in of finished tiles
      // Unit (tile, ks) of this CTA owns rows ks, ks + S_K, ... of the tile;
      // its rows are dealt round-robin to the kRowWarps warps.  A row waits
      // until all S_K units of its tile have stored their partials, then
      // reads x a second time -- from L2, about one round of units after
      // W0 brought it in.
      const int rw = warp - kRow0;
      rowdot::FwdRow<n> k;
      k.load(p.rows, lane);
      const int per_unit = (kBM + p.S_K - 1) / p.S_K;
      const int target = kUnitSignals * p.S_K;
      int item = 0, lu = 0;
      bool stop = false;
      for (int u = blockIdx.x; u < p.num_units && !stop; u += gridDim.x, ++lu) {
        const int tile = u / p.S_K, ks = u - (u / p.S_K) * p.S_K;
        bool ready = false;
        for (int m = 0; m < per_unit; ++m, ++item) {
          if (item % kRowWarps != rw) continue;
          const int r = ks + p.S_K * m;
          const int64_t t = (int64_t)tile * kBM + r;
          if (r >= kBM || t >= p.T) continue;
          if (!ready) {
            int ok = 0;
            if (lane == 0) ok = counter_wait(p.tile_done + tile, target, wc) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
              stop = true;
              break;
            }
            (void)ld_acquire(p.tile_done + tile);   // every lane acquires the partials' stores
            ready = true;
          }
          rowdot::fwd_row_token<n, kFp8, fused_row_chunks(n, kFp8)>(p.rows, k, t, lane);
        }
        if (lane == 0) rows_done[rw] = lu + 1;
      }
      if (lane == 0) rows_done[rw] = 1 << 30;   // done (or stopped): never hold W0 back again
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cf::TMEM_COLS);
  }
}

// phi [N_OUT, nD] f32 -> phis [NB, nD] bf16: rows t*N_OUT + j hold the t-th
// bf16 term of phi[j] (hi, mid, lo: each term rounds what the previous ones
// left), rows >= NT*N_OUT are zero.  With phi_bf16 given (phi unused) the
// rows are its bits: one exact term (NT = 1).  Also zeroes the fused
// forward's tile counters (tile_done may be null).
template <int n, int kNT = default_terms(n)>
__global__ void __launch_bounds__(256) split_phi_kernel(const float* __restrict__ phi,
                                                        const uint16_t* __restrict__ phi_bf16,
                                                        uint16_t* __restrict__ phis, int nD,
                                                        int* __restrict__ tile_done, int tiles) {
  // phis [NB][nD]: row term*N_OUT + j holds bf16 term `term` of phi[j]; rows
  // past NT*N_OUT are zero.  Each thread writes 8 consecutive k (one 16-byte
  // store); needs nD % 8 == 0.
  using Cf = Cfg<n, kNT>;
  if (tile_done)
    for (int64_t i = blockIdx.x * 256ll + threadIdx.x; i < tiles; i += (int64_t)gridDim.x * 256) MHC_ST(tile_done + i, 0);
  const int64_t per_row = nD / 8;
  const int64_t total = (int64_t)Cf::NB * per_row;
  for (int64_t idx = blockIdx.x * 256ll + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * 256) {
    const int r = (int)(idx / per_row);
    const int64_t k = (idx - (int64_t)r * per_row) * 8;
    uint32_t w[4] = {0, 0, 0, 0};
    if (phi_bf16 != nullptr) {
      if (r < Cf::N_OUT) {
        const uint4 v = MHC_LDG(reinterpret_cast<const uint4*>(phi_bf16 + (int64_t)r * nD + k));
        w[0] = v.x;
        w[1] = v.y;
        w[2] = v.z;
        w[3] = v.w;
      }
    } else if (r < Cf::NT * Cf::N_OUT) {
      const int term = r / Cf::N_OUT, j = r - term * Cf::N_OUT;
      const float4 a = MHC_LDG(reinterpret_cast<const float4*>(phi + (int64_t)j * nD + k));
      const float4 b = MHC_LDG(reinterpret_cast<const float4*>(phi + (int64_t)j * nD + k + 4));
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
    MHC_ST(reinterpret_cast<uint4*>(phis + (int64_t)r * nD + k), make_uint4(w[0], w[1], w[2], w[3]));
  }
}

}  // namespace fwdtc
}  // namespace mhc
