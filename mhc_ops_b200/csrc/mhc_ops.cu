// libmhc_ops: C-ABI entry points of the B200 mHC pre-op (declared in include/mhc_ops.h).
//
// Validation, workspace carving and kernel selection live here; the kernels
// are in generic.cuh (any shape), fwd_sm100.cuh / bwd_sm100.cuh (tcgen05 +
// TMA kernels for the shapes the tensor cores take), rowdot.cuh (the
// streaming whole-row kernels beside them), tiled.cuh (the backward for n
// other than 4) and post.cuh (the post-op that consumes h_post / h_res).

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <string>

#include <map>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "generic.cuh"
#include "sm100.cuh"
#include "fwd_sm100.cuh"
#include "bwd_sm100.cuh"
#include "rowdot.cuh"
#include "tiled.cuh"
#include "post.cuh"

#undef MHC_FILE_ID
#define MHC_FILE_ID 7   // debug-bounds site ids: 7 * 100000 + line

namespace mhc {

std::atomic<uint64_t> g_launch_count{0};
static thread_local std::string t_last_cuda_error;

void set_last_cuda_error(cudaError_t e) {
  t_last_cuda_error = std::string(cudaGetErrorName(e)) + ": " + cudaGetErrorString(e);
}

namespace {

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

template <template <int> class F, typename... Args>
int dispatch_n(int n, Args&&... args) {
  switch (n) {
    case 1: return F<1>::run(args...);
    case 2: return F<2>::run(args...);
    case 3: return F<3>::run(args...);
    case 4: return F<4>::run(args...);
    case 5: return F<5>::run(args...);
    case 6: return F<6>::run(args...);
    case 7: return F<7>::run(args...);
    case 8: return F<8>::run(args...);
    default: return MHC_ERR_BAD_SHAPE;
  }
}

int check_shape(int64_t T, int32_t n, int32_t D) {
  if (T < 0 || n < 1 || n > 8 || D < 1) return MHC_ERR_BAD_SHAPE;
  // Keep every element index inside int64 and every per-token row inside int32.
  if ((int64_t)n * D > (int64_t)1 << 28) return MHC_ERR_BAD_SHAPE;
  if (T > ((int64_t)1 << 40) / ((int64_t)n * D)) return MHC_ERR_BAD_SHAPE;
  return MHC_OK;
}

int current_sm_count(int* sms) {
  int dev = 0;
  MHC_CUDA_TRY(cudaGetDevice(&dev));
  int major = 0;
  MHC_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  if (major != 10) return MHC_ERR_NO_DEVICE;
  MHC_CUDA_TRY(cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev));
  return MHC_OK;
}

// ----------------------------------------------------------------- workspace
// Backward (generic path) workspace after the header:
//   dh_mix   [T][N]        f32
//   tokpart  [T][3+N]      f32   per-token dalpha / dbias terms
//   gpart    [P][N][nD]    f32   token-split partial sums of dh_mix^T x
struct BwdGenericLayout {
  size_t dh_mix, tokpart, gpart, total;
  int P;
  int64_t tokens_per_split;
};

BwdGenericLayout bwd_generic_layout(int64_t T, int n, int D, int sms) {
  BwdGenericLayout L{};
  const int N = n * n + 2 * n;
  const int64_t nD = (int64_t)n * D;
  const int64_t kblocks = (nD + generic::kThreads - 1) / generic::kThreads;
  int64_t P = std::max<int64_t>(1, (4 * (int64_t)sms + kblocks - 1) / kblocks);
  P = std::min<int64_t>(P, std::max<int64_t>(1, (T + 63) / 64));
  P = std::min<int64_t>(P, 256);
  L.P = (int)P;
  L.tokens_per_split = T > 0 ? (T + P - 1) / P : 1;
  size_t off = kWsHeaderBytes;
  L.dh_mix = off;
  off = align_up(off + sizeof(float) * (size_t)T * N, kWsAlign);
  L.tokpart = off;
  off = align_up(off + sizeof(float) * (size_t)T * (3 + N), kWsAlign);
  L.gpart = off;
  off = align_up(off + sizeof(float) * (size_t)P * N * nD, kWsAlign);
  L.total = off;
  return L;
}

// ----------------------------------------------------------------- generic runners
// Options of mhc_fwd_ex (all off for mhc_fwd): phi given as bf16 instead of
// fp32; the per-token RMSNorm factor of h_in for the next sublayer.
struct FwdEx {
  const uint16_t* phi_bf16 = nullptr;
  float* h_in_rstd = nullptr;
  float h_in_eps = 0.f;
  int sm_budget = 0;               // > 0: grids use at most this many SMs
  const uint8_t* x_fp8 = nullptr;  // x as e4m3 bytes (then args->x is unused) ...
  const int8_t* x_exp = nullptr;   // ... times 2^x_exp[t] per token
};

template <int n>
struct FwdGeneric {
  static int run(const mhc_fwd_args* a, const float* phi, const FwdEx& ex, cudaStream_t s, int sms) {
    const int64_t T = a->tokens;
    const int grid = (int)std::min<int64_t>(T, (int64_t)sms * 8);
    generic::fwd_kernel<n><<<grid, generic::kThreads, 0, s>>>(
        a->x, phi, a->alpha, a->bias, a->h_in, a->h_post, a->h_res, a->inv_rms, a->h_mix, a->h_pre, T,
        a->D, a->norm_eps, a->hc_eps, ex.h_in_rstd, ex.h_in_eps);
    return after_launch();
  }
};

// bf16 phi -> an fp32 copy, for the generic forward (exact widening).
__global__ void phi_widen_kernel(const uint16_t* __restrict__ src, float* __restrict__ dst, int64_t count) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    MHC_ST(dst + i, bf16_bits_to_f32(MHC_LD(src + i)));
}

template <int n>
struct BwdGeneric {
  static int run(const mhc_bwd_args* a, cudaStream_t s, int sms) {
    constexpr int N = n * n + 2 * n;
    const int64_t T = a->tokens;
    const int nD = n * a->D;
    BwdGenericLayout L = bwd_generic_layout(T, n, a->D, sms);
    char* ws = static_cast<char*>(a->workspace);
    float* dh_mix = reinterpret_cast<float*>(ws + L.dh_mix);
    float* tokpart = reinterpret_cast<float*>(ws + L.tokpart);
    float* gpart = reinterpret_cast<float*>(ws + L.gpart);
    const int grid = (int)std::min<int64_t>(T, (int64_t)sms * 8);
    generic::bwd_token_kernel<n><<<grid, generic::kThreads, 0, s>>>(
        a->x, a->phi, a->alpha, a->inv_rms, a->h_mix, a->h_pre, a->h_post, a->dh_in, a->dh_post, a->dh_res,
        a->gamma, a->dx, dh_mix, tokpart, T, a->D, a->hc_eps);
    int st = after_launch();
    if (st) return st;
    dim3 g2((nD + generic::kThreads - 1) / generic::kThreads, L.P);
    generic::bwd_g_kernel<n><<<g2, generic::kThreads, 0, s>>>(a->x, dh_mix, gpart, T, nD, L.tokens_per_split);
    if ((st = after_launch())) return st;
    generic::finalize_param_kernel<N><<<(nD + generic::kFinCols - 1) / generic::kFinCols + 3 + N, generic::kThreads, 0,
                                        s>>>(gpart, L.P, a->phi, a->gamma, a->dphi, a->dgamma, nD, tokpart, T, a->dalpha,
                                             a->dbias);
    return after_launch();
  }
};

// ----------------------------------------------------------------- driver entry points, TMA maps
// A CUDA driver function looked up through the runtime (NULL if unavailable).
void* driver_entry_point(const char* name) {
  void* ptr = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    ptr = nullptr;
  return ptr;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn =
      reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(driver_entry_point("cuTensorMapEncodeTiled"));
  return fn;
}

// Row-major tensor of `rank` dims (dims[0] innermost) -> tiled TMA map.  L2
// promotion is 128 bytes, the width of every box row here: with 256-byte
// promotion the neighbouring lines are evicted before their own box asks for
// them (measured on B200: the backward kernel then reads ~39% more than it
// needs; an L2 prefetch of its boxes 8 stages ahead wastes reads the same way).
int encode_map(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  auto enc = tensor_map_encoder();
  if (!enc) return MHC_ERR_CUDA;
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUresult r = enc(map, dtype, rank, const_cast<void*>(base), d, st, b, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MHC_OK : MHC_ERR_CUDA;
}

int encode_bf16_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                    const uint32_t* box, CUtensorMapSwizzle swz) {
  return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, rank, dims, strides_bytes, box, swz);
}

// ----------------------------------------------------------------- launch helpers
// Raise a kernel's dynamic shared memory limit once per (device, kernel).
template <typename Kernel>
int set_smem_limit_once(Kernel kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  MHC_CUDA_TRY(cudaGetDevice(&dev));
  const auto key = std::make_pair(dev, reinterpret_cast<const void*>(kernel));
  std::lock_guard<std::mutex> lk(mu);
  if (done.count(key)) return MHC_OK;
  MHC_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.insert(key);
  return MHC_OK;
}

// ----------------------------------------------------------------- tensor-core forward
// fwdtc::proj_kernel (tcgen05 projection -> per (token, K-slice) partial rows,
// parked in the token's h_in row) and the row half (gates, outputs, h_in),
// either fused into one cooperative launch (proj_kernel<n, true>: row warps
// follow the projection tile by tile through per-tile counters, so x's second
// read hits L2) or as a second kernel (rowdot::fwd_rows_kernel) when the
// fused form's finer K-slices do not fit in an h_in row or the device cannot
// co-schedule its grid.  Shapes they take: any n, D a multiple of 64 whose
// h_in row holds at least one partial row (n = 8: D >= 192), 16-byte aligned
// x / h_in / phi, T < 2^31; the fused form n = 4 only, an fp8 x n in {4, 8}.
// Everything else runs the generic kernels.
template <int n>
struct FwdPartRowBytes {
  static int run() { return 4 * fwdtc::Cfg<n>::RW; }
};
int fwd_part_row_bytes(int n) { return dispatch_n<FwdPartRowBytes>(n); }

bool fwd_tc_shape(int64_t T, int n, int D) {
  if (n < 1 || n > 8) return false;
  if (D % 64 != 0 || T >= ((int64_t)1 << 31)) return false;
  return 2 * D >= fwd_part_row_bytes(n);
}

bool fwd_tc_eligible(const mhc_fwd_args* a, const FwdEx& ex) {
  const void* phi = ex.phi_bf16 ? static_cast<const void*>(ex.phi_bf16) : static_cast<const void*>(a->phi);
  const void* x = ex.x_fp8 ? static_cast<const void*>(ex.x_fp8) : static_cast<const void*>(a->x);
  return fwd_tc_shape(a->tokens, a->n, a->D) && aligned(x, 16) && aligned(a->h_in, 16) && aligned(phi, 16);
}

// Bytes of the bf16 term images of phi (one term when phi comes in bf16).
template <int n>
struct FwdTermRows {
  static int run(bool bf16_phi) { return bf16_phi ? fwdtc::Cfg<n, 1>::NB : fwdtc::Cfg<n>::NB; }
};
size_t fwd_tc_phis_bytes(int n, int D, bool bf16_phi) {
  const int NB = dispatch_n<FwdTermRows>(n, bf16_phi);
  return (size_t)NB * n * D * sizeof(uint16_t);
}

struct FwdTcPlan {
  bool fused = false;
  int S_K = 1;      // K-slices
  int KB_PER = 1;   // 64-wide K-blocks per slice
  int units = 1;    // tiles * S_K
  int grid = 1;     // persistent CTAs of proj_kernel
};

// Fused forward: a unit is at most this many K-blocks (128 KB of x), so one
// round of units over all SMs reads ~20 MB and x is still in L2 when the row
// warps read it again (measured on B200: a 256 KB block per SM survives ~55 MB
// of other traffic, and misses after ~75 MB).
constexpr int kFusedKbPer = 8;

// K-slices of the fused forward: the fewest (a divisor of the n*D/64
// K-blocks, at most 128) with units of at most kFusedKbPer K-blocks; 0 when
// that many partial rows do not fit in an h_in row.
int fwd_fused_slices(int n, int D) {
  const int KB = n * D / fwdtc::kBK;
  for (int sk = 1; sk <= std::min(KB, fwdtc::kBM); ++sk) {
    if (KB % sk != 0 || KB / sk > kFusedKbPer) continue;
    return sk * fwd_part_row_bytes(n) <= 2 * D ? sk : 0;
  }
  return 0;
}

// Whether proj_kernel<n, true, NT> can run with one CTA on every SM at once
// (a cooperative launch needs that); asked once per device.
template <int n, int NT, bool FP8 = false>
bool fwd_fused_supported() {
  static std::mutex mu;
  static std::map<int, bool> known;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lk(mu);
  auto it = known.find(dev);
  if (it != known.end()) return it->second;
  int coop = 0, blocks = 0;
  bool ok = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) == cudaSuccess && coop &&
            cudaFuncSetAttribute(fwdtc::proj_kernel<n, true, NT, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 fwdtc::Cfg<n, NT, FP8>::SMEM) == cudaSuccess &&
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fwdtc::proj_kernel<n, true, NT, FP8>,
                                                          fwdtc::threads_of(true, FP8),
                                                          fwdtc::Cfg<n, NT, FP8>::SMEM) == cudaSuccess &&
            blocks >= 1;
  (void)cudaGetLastError();
  known[dev] = ok;
  return ok;
}

// n = 8 never qualifies (its K-slices of at most kFusedKbPer blocks need more
// partial rows than an h_in row holds), so only n = 4 is instantiated.
bool fwd_fused_supported(int n, bool bf16_phi = false, bool fp8_x = false) {
  if (n != 4) return false;
  if (fp8_x) return bf16_phi ? fwd_fused_supported<4, 1, true>() : fwd_fused_supported<4, 3, true>();
  return bf16_phi ? fwd_fused_supported<4, 1>() : fwd_fused_supported<4, fwdtc::default_terms(4)>();
}

// Two-kernel form: the fewest K-slices (a divisor of the n*D/64 K-blocks, at
// most 16, and no more than an h_in row holds) that give every SM at least
// ~4 units.  Fused form: fwd_fused_slices, one CTA per SM at most.
// fused_ok: whether the fused form's cooperative launch fits on the device
// (fwd_fused_supported; true on every sm_100 part for n = 4).
FwdTcPlan fwd_tc_plan_with(int64_t T, int n, int D, int sms, bool fused_ok) {
  FwdTcPlan P;
  const int KB = n * D / fwdtc::kBK;
  const int64_t tiles = std::max<int64_t>(1, (T + fwdtc::kBM - 1) / fwdtc::kBM);
  const int fused_sk = fwd_fused_slices(n, D);
  if (fused_sk > 0 && fused_ok) {
    P.fused = true;
    P.S_K = fused_sk;
  } else {
    const int max_sk = std::min(16, 2 * D / fwd_part_row_bytes(n));
    for (int sk = 1; sk <= max_sk; ++sk) {
      if (KB % sk != 0) continue;
      P.S_K = sk;
      if (tiles * sk >= 4 * (int64_t)sms) break;
    }
  }
  P.KB_PER = KB / P.S_K;
  P.units = (int)(tiles * P.S_K);
  P.grid = std::min(P.units, sms);
  return P;
}

FwdTcPlan fwd_tc_plan(int64_t T, int n, int D, int sms, bool bf16_phi, bool fp8_x) {
  return fwd_tc_plan_with(T, n, D, sms, fwd_fused_supported(n, bf16_phi, fp8_x));
}

size_t fwd_tile_counter_bytes(int64_t T) {
  return sizeof(int) * (size_t)std::max<int64_t>(1, (T + fwdtc::kBM - 1) / fwdtc::kBM);
}

int fwd_rows_grid(int64_t T, int sms) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(sms, (T + rowdot::kWarps - 1) / rowdot::kWarps));
}

template <int n, int NT, bool FP8>
struct FwdTc {
  // One cooperative launch of proj_kernel<n, true, NT> (all CTAs co-resident:
  // row warps wait on counters other CTAs advance).
  static int launch_fused(const CUtensorMap& m_x2d, const CUtensorMap& m_phi, const fwdtc::Params& p,
                          const FwdTcPlan& P, cudaStream_t s) {
    using Cf = fwdtc::Cfg<n, NT, FP8>;
    int st;
    if ((st = set_smem_limit_once(fwdtc::proj_kernel<n, true, NT, FP8>, Cf::SMEM))) return st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P.grid);
    cfg.blockDim = dim3(fwdtc::threads_of(true, FP8));
    cfg.dynamicSmemBytes = Cf::SMEM;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    MHC_CUDA_TRY(cudaLaunchKernelEx(&cfg, fwdtc::proj_kernel<n, true, NT, FP8>, m_x2d, m_phi, p));
    return after_launch();
  }

  static int run(const mhc_fwd_args* a, const FwdEx& ex, cudaStream_t s, int sms) {
    using Cf = fwdtc::Cfg<n, NT, FP8>;
    const bool bf16_phi = ex.phi_bf16 != nullptr;
    const int64_t T = a->tokens;
    const int D = a->D;
    const int nD = n * D;
    char* ws = static_cast<char*>(a->workspace);
    uint16_t* phis = reinterpret_cast<uint16_t*>(ws + kWsHeaderBytes);
    int* tile_done =
        reinterpret_cast<int*>(ws + align_up(kWsHeaderBytes + fwd_tc_phis_bytes(n, D, bf16_phi), kWsAlign));
    const FwdTcPlan P = fwd_tc_plan(T, n, D, sms, bf16_phi, FP8);
    const int tiles = (int)((T + fwdtc::kBM - 1) / fwdtc::kBM);
    int st;

    fwdtc::split_phi_kernel<n, NT>
        <<<std::min<int64_t>(((int64_t)Cf::NB * nD / 8 + 255) / 256, 4 * 148), 256, 0, s>>>(
            a->phi, ex.phi_bf16, phis, nD, P.fused ? tile_done : nullptr, tiles);
    if ((st = after_launch())) return st;

    CUtensorMap m_x2d, m_phi;
    {
      const uint64_t dims[2] = {(uint64_t)nD, (uint64_t)T};
      const uint64_t strides[1] = {(uint64_t)nD * 2};
      const uint32_t box[2] = {fwdtc::kBK, fwdtc::kBM};
      if constexpr (FP8) {
        // [128 tok x 64 k] e4m3 bytes, unswizzled: the sum-of-squares warps
        // read their row of it and write the swizzled bf16 tile
        const uint64_t strides8[1] = {(uint64_t)nD};
        if ((st = encode_map(&m_x2d, CU_TENSOR_MAP_DATA_TYPE_UINT8, ex.x_fp8, 2, dims, strides8, box,
                             CU_TENSOR_MAP_SWIZZLE_NONE)))
          return st;
      } else {
        if ((st = encode_bf16_map(&m_x2d, a->x, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
      }
    }
    {
      const uint64_t dims[2] = {(uint64_t)nD, (uint64_t)Cf::NB};
      const uint64_t strides[1] = {(uint64_t)nD * 2};
      const uint32_t box[2] = {fwdtc::kBK, (uint32_t)Cf::NB};
      if ((st = encode_bf16_map(&m_phi, phis, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    }
    fwdtc::Params p;
    p.part = reinterpret_cast<float*>(a->h_in);
    p.part_stride = D / 2;
    p.status = reinterpret_cast<int*>(ws);
    p.T = T;
    p.S_K = P.S_K;
    p.KB_PER = P.KB_PER;
    p.num_units = P.units;
    p.tile_done = tile_done;
    p.rows.x = a->x;
    p.rows.alpha = a->alpha;
    p.rows.bias = a->bias;
    p.rows.h_in = a->h_in;
    p.rows.h_post = a->h_post;
    p.rows.h_res = a->h_res;
    p.rows.inv_rms = a->inv_rms;
    p.rows.h_mix = a->h_mix;
    p.rows.h_pre = a->h_pre;
    p.rows.D = D;
    p.rows.S_K = P.S_K;
    p.rows.RW = Cf::RW;
    p.rows.h_in_rstd = ex.h_in_rstd;
    p.rows.x8 = ex.x_fp8;
    p.rows.x_exp = ex.x_exp;
    p.rows.norm_eps = a->norm_eps;
    p.rows.hc_eps = a->hc_eps;
    p.rows.h_in_eps = ex.h_in_eps;
    if constexpr (n == 4) {
      if (P.fused) return launch_fused(m_x2d, m_phi, p, P, s);
    }
    if ((st = set_smem_limit_once(fwdtc::proj_kernel<n, false, NT, FP8>, Cf::SMEM))) return st;
    fwdtc::proj_kernel<n, false, NT, FP8><<<P.grid, fwdtc::kThreads, Cf::SMEM, s>>>(m_x2d, m_phi, p);
    if ((st = after_launch())) return st;
    rowdot::fwd_rows_kernel<n, FP8><<<fwd_rows_grid(T, sms), rowdot::kThreads, 0, s>>>(p.rows, T);
    return after_launch();
  }
};

// Header (status word), split-phi images, then the fused form's per-tile
// counters; with a bf16 phi, last, the fp32 copy the generic kernels read.
size_t fwd_phi_copy_offset(int64_t T, int n, int D, bool bf16_phi) {
  size_t b = kWsHeaderBytes;
  if (fwd_tc_shape(T, n, D)) {
    b = align_up(b + fwd_tc_phis_bytes(n, D, bf16_phi), kWsAlign);
    b = align_up(b + fwd_tile_counter_bytes(T), kWsAlign);
  }
  return b;
}

int fwd_workspace(int64_t T, int n, int D, size_t* bytes, bool bf16_phi = false) {
  size_t b = fwd_phi_copy_offset(T, n, D, bf16_phi);
  if (bf16_phi) b = align_up(b + sizeof(float) * (size_t)(n * n + 2 * n) * n * D, kWsAlign);
  *bytes = b;
  return MHC_OK;
}

// Tensor-core forward of a bf16 x for stream count n (one phi term when phi
// comes in bf16).
template <int n>
struct FwdTcBf16 {
  static int run(const mhc_fwd_args* a, const FwdEx& ex, cudaStream_t s, int sms) {
    return ex.phi_bf16 ? FwdTc<n, 1, false>::run(a, ex, s, sms)
                       : FwdTc<n, fwdtc::default_terms(n), false>::run(a, ex, s, sms);
  }
};

// The forward, any shape (arguments already validated).
int fwd_run(const mhc_fwd_args* a, const FwdEx& ex, cudaStream_t s, int sms) {
  const bool bf16_phi = ex.phi_bf16 != nullptr;
  if (fwd_tc_eligible(a, ex)) {
    if (ex.x_fp8) {
      if (a->n == 4) return bf16_phi ? FwdTc<4, 1, true>::run(a, ex, s, sms) : FwdTc<4, 3, true>::run(a, ex, s, sms);
      if (a->n == 8) return bf16_phi ? FwdTc<8, 1, true>::run(a, ex, s, sms) : FwdTc<8, 2, true>::run(a, ex, s, sms);
      return MHC_ERR_BAD_SHAPE;
    }
    return dispatch_n<FwdTcBf16>(a->n, a, ex, s, sms);
  }
  if (ex.x_fp8) return MHC_ERR_BAD_SHAPE;   // fp8 x: tensor-core shapes only
  const float* phi = a->phi;
  if (bf16_phi) {
    float* copy = reinterpret_cast<float*>(static_cast<char*>(a->workspace) +
                                           fwd_phi_copy_offset(a->tokens, a->n, a->D, true));
    const int64_t count = (int64_t)(a->n * a->n + 2 * a->n) * a->n * a->D;
    phi_widen_kernel<<<(int)std::min<int64_t>((count + 255) / 256, 4 * (int64_t)sms), 256, 0, s>>>(ex.phi_bf16, copy,
                                                                                                  count);
    int st = after_launch();
    if (st) return st;
    phi = copy;
  }
  return dispatch_n<FwdGeneric>(a->n, a, phi, ex, s, sms);
}

// ----------------------------------------------------------------- tensor-core backward
// Two kernels: rowdot::bwd_rows_kernel (whole-row reductions -> one record
// per token) and bwdtc::bwd_kernel (tcgen05 GEMMs over the records, CTA =
// d-slice x token group).  Shapes they take: n == 4, D a multiple of 64,
// 16-byte aligned x / dh_in / dx / phi, T < 2^31.
constexpr int kBwdN = 4;
constexpr int kRowsWarps = rowdot::kWarps;

struct BwdTcPlan {
  int Dc = 0;     // d-slice width
  int S_K = 0;    // d-slices
  int S_T = 0;    // token groups
  // Leftover tiles: with E > 0 the S_K * S_T main CTAs take J tiles each
  // (tiles R .. tiles-1) and E more CTAs take the R leftover tiles (0 .. R-1)
  // of ES whole d-slices each, so no CTA does more than max(J, R * ES) units
  // of (tile, d-slice).  E = 0: the main CTAs share every tile round robin.
  int J = 0;
  int E = 0;
  int ES = 0;
  int R = 0;
  int ctas() const { return S_K * S_T + E; }
  int gpart_slots() const { return S_T + (E > 0 ? 1 : 0); }
};

struct BwdTcLayout {
  size_t phit, rec, gpart, abpart, total;
  BwdTcPlan plan;
  int rows_grid;  // CTAs of the row kernel
};

// Slice width Dc (multiple of 64 dividing D, n*Dc <= MAX_KC) with the least
// per-CTA work in units of (tile, d-slice) times Dc; S_T = sms / S_K token
// groups.  Round robin: waves * ceil(tiles / S_T) units for the busiest CTA.
// With SMs to spare (sms > S_K * S_T) and tiles % S_T = R > 0, the leftover
// tiles may go to E' extra CTAs instead (E' the largest divisor of S_K that
// fits, so each takes whole d-slices and owns its slot of the G partials):
// max(tiles / S_T, R * S_K / E') units.  Ties go to the wider slice (fewer,
// longer CTAs), then to round robin.
BwdTcPlan bwd_tc_plan(int64_t T, int D, int sms) {
  using Cf = bwdtc::Cfg<kBwdN>;
  const int64_t tiles = std::max<int64_t>(1, (T + bwdtc::kBM - 1) / bwdtc::kBM);
  BwdTcPlan best;
  double best_cost = 0.0;
  for (int Dc = 64; Dc * kBwdN <= Cf::MAX_KC; Dc += 64) {
    if (D % Dc != 0) continue;
    const int S_K = D / Dc;
    const int64_t S_T = std::min<int64_t>(std::max(1, sms / S_K), tiles);
    const int64_t waves = ((int64_t)S_K * S_T + sms - 1) / sms;
    BwdTcPlan cand{Dc, S_K, (int)S_T};
    double cost = (double)waves * (double)((tiles + S_T - 1) / S_T) * Dc;
    const int64_t spare = (int64_t)sms - (int64_t)S_K * S_T;
    const int64_t R = tiles % S_T;
    if (waves == 1 && spare > 0 && R > 0) {
      int Ex = 0;
      for (int e = 1; e <= spare && e <= S_K; ++e)
        if (S_K % e == 0) Ex = e;
      const int64_t J = tiles / S_T;
      const int64_t extra_units = R * (S_K / Ex);
      const double bal = (double)std::max(J, extra_units) * Dc;
      if (bal < cost - 1e-9) {
        cand.J = (int)J;
        cand.E = Ex;
        cand.ES = S_K / Ex;
        cand.R = (int)R;
        cost = bal;
      }
    }
    if (best.Dc == 0 || cost <= best_cost + 1e-9) {
      best = cand;
      best_cost = cost;
    }
  }
  return best;
}

rowdot::BwdRowArgs bwd_row_args(const mhc_bwd_args* a, float* rec) {
  rowdot::BwdRowArgs r;
  r.x = a->x;
  r.dh_in = a->dh_in;
  r.alpha = a->alpha;
  r.inv_rms = a->inv_rms;
  r.h_mix = a->h_mix;
  r.h_pre = a->h_pre;
  r.h_post = a->h_post;
  r.dh_post = a->dh_post;
  r.dh_res = a->dh_res;
  r.rec = rec;
  r.D = a->D;
  r.hc_eps = a->hc_eps;
  r.img_phi = nullptr;
  r.img_gamma = nullptr;
  r.img = nullptr;
  r.img_blocks = 0;
  return r;
}

// The row kernel's arguments with the split phi * gamma images to build into
// img (one warp per 64-k block, before its tokens): the layout of
// bwdtc::Cfg<4> / tiled::DxCfg<n> (3 term segments of round_up(N, 16) columns).
rowdot::BwdRowArgs bwd_row_args_with_image(const mhc_bwd_args* a, float* rec, uint8_t* img) {
  rowdot::BwdRowArgs r = bwd_row_args(a, rec);
  r.img_phi = a->phi;
  r.img_gamma = a->gamma;
  r.img = img;
  r.img_blocks = a->n * a->D / 64;
  return r;
}

int bwd_rows_grid(int64_t T, int sms) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(sms, (T + kRowsWarps - 1) / kRowsWarps));
}

BwdTcLayout bwd_tc_layout(int64_t T, int D, int sms) {
  using Cf = bwdtc::Cfg<kBwdN>;
  BwdTcLayout L{};
  L.plan = bwd_tc_plan(T, D, sms);
  L.rows_grid = bwd_rows_grid(T, sms);
  const int64_t nD = (int64_t)kBwdN * D;
  size_t off = kWsHeaderBytes;
  L.phit = off;
  off = align_up(off + (size_t)(nD / 64) * Cf::PH_BYTES, kWsAlign);
  L.rec = off;
  off = align_up(off + sizeof(float) * (size_t)T * Cf::RECW, kWsAlign);
  L.gpart = off;
  off = align_up(off + sizeof(float) * (size_t)L.plan.gpart_slots() * Cf::N_OUT * nD, kWsAlign);
  L.abpart = off;
  off = align_up(off + sizeof(float) * (size_t)L.rows_grid * kRowsWarps * Cf::CW, kWsAlign);
  L.total = off;
  return L;
}

bool bwd_tc_shape(int64_t T, int n, int D) {
  return n == kBwdN && D % 64 == 0 && T < ((int64_t)1 << 31);
}

bool bwd_tc_eligible(const mhc_bwd_args* a) {
  return bwd_tc_shape(a->tokens, a->n, a->D) && aligned(a->x, 16) && aligned(a->dh_in, 16) &&
         aligned(a->dx, 16) && aligned(a->phi, 16);
}

int bwd_tc_run(const mhc_bwd_args* a, cudaStream_t s, int sms) {
  using Cf = bwdtc::Cfg<kBwdN>;
  constexpr int n = kBwdN;
  static_assert(rowdot::Rec<n>::W == Cf::RECW && rowdot::Rec<n>::CW == Cf::CW, "record layouts differ");
  const int64_t T = a->tokens;
  const int D = a->D;
  const int nD = n * D;
  const BwdTcLayout L = bwd_tc_layout(T, D, sms);
  char* ws = static_cast<char*>(a->workspace);
  float* rec = reinterpret_cast<float*>(ws + L.rec);
  float* gpart = reinterpret_cast<float*>(ws + L.gpart);
  float* abpart = reinterpret_cast<float*>(ws + L.abpart);
  const int num_tiles = (int)((T + bwdtc::kBM - 1) / bwdtc::kBM);
  int st;

  static_assert(Cf::KA == 3 * ((Cf::N_OUT + 15) / 16 * 16) && Cf::PH_BYTES == 8 * (Cf::KA / 8) * 128,
                "phi images as rowdot::split_image_block lays them out");
  rowdot::bwd_rows_kernel<n><<<L.rows_grid, rowdot::kThreads, 0, s>>>(
      bwd_row_args_with_image(a, rec, reinterpret_cast<uint8_t*>(ws + L.phit)), abpart, T);
  if ((st = after_launch())) return st;

  CUtensorMap m_x2d, m_dh, m_dx, m_rec;
  {
    const uint64_t dims[2] = {(uint64_t)nD, (uint64_t)T};
    const uint64_t strides[1] = {(uint64_t)nD * 2};
    const uint32_t box[2] = {bwdtc::kBK, bwdtc::kBM};
    if ((st = encode_bf16_map(&m_x2d, a->x, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
    if ((st = encode_bf16_map(&m_dx, a->dx, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)D, (uint64_t)T};
    const uint64_t strides[1] = {(uint64_t)D * 2};
    const uint32_t box[2] = {bwdtc::kBK, bwdtc::kBM};
    if ((st = encode_bf16_map(&m_dh, a->dh_in, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)Cf::RECW, (uint64_t)T};
    const uint64_t strides[1] = {(uint64_t)Cf::RECW * 4};
    const uint32_t box[2] = {(uint32_t)Cf::RECW, bwdtc::kBM};
    if ((st = encode_map(&m_rec, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rec, 2, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_128B)))
      return st;
  }
  bwdtc::Params p;
  p.phit = reinterpret_cast<const uint8_t*>(ws + L.phit);
  p.gpart = gpart;
  p.status = reinterpret_cast<int*>(ws);
  p.T = T;
  p.D = D;
  p.Dc = L.plan.Dc;
  p.S_K = L.plan.S_K;
  p.S_T = L.plan.S_T;
  p.J = L.plan.J;
  p.E = L.plan.E;
  p.ES = L.plan.ES;
  p.R = L.plan.R;
  p.num_tiles = num_tiles;

  if ((st = set_smem_limit_once(bwdtc::bwd_kernel<n>, Cf::SMEM))) return st;
  bwdtc::bwd_kernel<n><<<L.plan.ctas(), bwdtc::kThreads, Cf::SMEM, s>>>(m_x2d, m_dh, m_dx, m_rec, p);
  if ((st = after_launch())) return st;

  generic::finalize_param_kernel<Cf::N_OUT>
      <<<(nD + generic::kFinCols - 1) / generic::kFinCols + 3 + Cf::N_OUT, generic::kThreads, 0, s>>>(
          gpart, L.plan.gpart_slots(), a->phi, a->gamma, a->dphi, a->dgamma, nD, abpart, (int64_t)L.rows_grid * kRowsWarps,
          a->dalpha, a->dbias);
  return after_launch();
}

// ----------------------------------------------------------------- tiled backward (n != 4)
// rowdot::bwd_rows_kernel (records and the split phi images), dx (dx_tc_kernel
// on the tensor cores, or transpose_kernel + dx_kernel on the CUDA cores),
// tiled::gimg_kernel + g_tc_kernel (tcgen05), then the shared finalize kernel.  Shapes: every n the tensor-core backward does
// not take, D a multiple of 8, 16-byte aligned x / dh_in / dx / phi / gamma,
// T < 2^31.
struct BwdTiledLayout {
  size_t rec, abpart, gpart, gimg, dmT, phimg, total;
  bool dx_tc;            // dx on the tensor cores (D % 64 == 0), else dx_kernel
  bool dx_pair;          // even n: dx_tc_pair_kernel (pairs of 64-k blocks), else dx_tc_kernel
  int dx_slices;         // unit ranges per token tile
  int dx_kb_per;         // units (64-k blocks, or pairs) per range
  int P;                 // token groups of the G partials (g_tc_kernel's grid.y)
  int rows_grid;
};

int rec_width(int n) {
  const int N = n * n + 2 * n;
  return ((N + 1 + n) + 3) / 4 * 4;
}

size_t bwd_tiled_phimg_bytes(int n) {
  switch (n) {
    case 1: return tiled::DxCfg<1>::PH_BYTES;
    case 2: return tiled::DxCfg<2>::PH_BYTES;
    case 3: return tiled::DxCfg<3>::PH_BYTES;
    case 4: return tiled::DxCfg<4>::PH_BYTES;
    case 5: return tiled::DxCfg<5>::PH_BYTES;
    case 6: return tiled::DxCfg<6>::PH_BYTES;
    case 7: return tiled::DxCfg<7>::PH_BYTES;
    default: return tiled::DxCfg<8>::PH_BYTES;
  }
}

size_t bwd_tiled_gimg_bytes(int n) {
  switch (n) {
    case 1: return tiled::GCfg<1>::DHM_BYTES;
    case 2: return tiled::GCfg<2>::DHM_BYTES;
    case 3: return tiled::GCfg<3>::DHM_BYTES;
    case 4: return tiled::GCfg<4>::DHM_BYTES;
    case 5: return tiled::GCfg<5>::DHM_BYTES;
    case 6: return tiled::GCfg<6>::DHM_BYTES;
    case 7: return tiled::GCfg<7>::DHM_BYTES;
    default: return tiled::GCfg<8>::DHM_BYTES;
  }
}

BwdTiledLayout bwd_tiled_layout(int64_t T, int n, int D, int sms) {
  BwdTiledLayout L{};
  const int N = n * n + 2 * n;
  const int64_t nD = (int64_t)n * D;
  // token groups of the tensor-core G kernel: the fewest with the least
  // per-CTA work, waves * ceil(tiles / S_T), over ceil(nD / 128) k-ranges
  const int64_t kranges = (nD + 127) / 128;
  const int64_t tiles = std::max<int64_t>(1, (T + 127) / 128);
  int64_t best = 1;
  double best_cost = 0.0;
  // (at most 8 groups: the partial sums take S_T * N * nD floats; a larger
  // S_T must save at least 3% to be taken)
  for (int64_t st = 1; st <= std::min<int64_t>(tiles, 8); ++st) {
    const double cost = (double)((kranges * st + sms - 1) / sms) * (double)((tiles + st - 1) / st);
    if (st == 1 || cost < 0.97 * best_cost) {
      best = st;
      best_cost = cost;
    }
  }
  L.P = (int)best;
  L.rows_grid = bwd_rows_grid(T, sms);
  size_t off = kWsHeaderBytes;
  L.rec = off;
  off = align_up(off + sizeof(float) * (size_t)T * rec_width(n), kWsAlign);
  L.abpart = off;
  off = align_up(off + sizeof(float) * (size_t)L.rows_grid * kRowsWarps * (3 + N), kWsAlign);
  L.gpart = off;
  off = align_up(off + sizeof(float) * (size_t)L.P * N * nD, kWsAlign);
  L.gimg = off;
  off = align_up(off + (size_t)tiles * bwd_tiled_gimg_bytes(n), kWsAlign);
  L.dx_tc = D % 64 == 0;
  if (L.dx_tc) {
    // ranges of work units (64-k blocks; pairs of them for even n) per tile
    // with the least per-CTA work, waves * units per range
    const int64_t KB = nD / 64;
    L.dx_pair = n % 2 == 0;
    const int64_t units = L.dx_pair ? KB / 2 : KB;
    int64_t best_s = 1;
    double best_c = 0.0;
    for (int64_t sl = 1; sl <= std::min<int64_t>(units, 64); ++sl) {
      const double c = (double)((tiles * sl + sms - 1) / sms) * (double)((units + sl - 1) / sl);
      if (sl == 1 || c < best_c - 1e-9) {
        best_s = sl;
        best_c = c;
      }
    }
    L.dx_slices = (int)best_s;
    L.dx_kb_per = (int)((units + best_s - 1) / best_s);
    L.phimg = off;
    off = align_up(off + (size_t)KB * bwd_tiled_phimg_bytes(n), kWsAlign);
  } else {
    L.dmT = off;
    off = align_up(off + sizeof(float) * (size_t)N * tiled::padded_tokens(T), kWsAlign);
  }
  L.total = off;
  return L;
}

bool bwd_tiled_shape(int64_t T, int n, int D) {
  return n >= 1 && n <= 8 && D % 8 == 0 && T < ((int64_t)1 << 31);
}

bool bwd_tiled_eligible(const mhc_bwd_args* a) {
  return bwd_tiled_shape(a->tokens, a->n, a->D) && aligned(a->x, 16) && aligned(a->dh_in, 16) &&
         aligned(a->dx, 16) && aligned(a->phi, 16) && aligned(a->gamma, 16);
}

template <int n>
struct BwdTiled {
  static int run(const mhc_bwd_args* a, cudaStream_t s, int sms) {
    using Dm = tiled::Dims<n>;
    constexpr int N = Dm::N;
    static_assert(Dm::RW == rowdot::Rec<n>::W && 3 + N == rowdot::Rec<n>::CW, "record layouts differ");
    const int64_t T = a->tokens;
    const int D = a->D;
    const int nD = n * D;
    const BwdTiledLayout L = bwd_tiled_layout(T, n, D, sms);
    char* ws = static_cast<char*>(a->workspace);
    float* rec = reinterpret_cast<float*>(ws + L.rec);
    float* abpart = reinterpret_cast<float*>(ws + L.abpart);
    float* gpart = reinterpret_cast<float*>(ws + L.gpart);
    int st;
    // dx on the tensor cores reads split phi * gamma images, which the row
    // kernel's warps build before their tokens
    static_assert(tiled::DxCfg<n>::KA == 3 * ((N + 15) / 16 * 16) &&
                      tiled::DxCfg<n>::PH_BYTES == 8 * (tiled::DxCfg<n>::KA / 8) * 128,
                  "phi images as rowdot::split_image_block lays them out");
    uint8_t* img = L.dx_tc ? reinterpret_cast<uint8_t*>(ws + L.phimg) : nullptr;
    rowdot::bwd_rows_kernel<n><<<L.rows_grid, rowdot::kThreads, 0, s>>>(
        img ? bwd_row_args_with_image(a, rec, img) : bwd_row_args(a, rec), abpart, T);
    if ((st = after_launch())) return st;
    if (L.dx_tc) {
      // dx on the tensor cores: one CTA per (token tile, range of 64-k blocks)
      using Dc = tiled::DxCfg<n>;
      CUtensorMap m_x, m_dh;
      {
        const uint64_t dims[2] = {(uint64_t)nD, (uint64_t)T};
        const uint64_t strides[1] = {(uint64_t)nD * 2};
        const uint32_t box[2] = {64, 128};
        if ((st = encode_bf16_map(&m_x, a->x, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
      }
      {
        const uint64_t dims[2] = {(uint64_t)D, (uint64_t)T};
        const uint64_t strides[1] = {(uint64_t)D * 2};
        const uint32_t box[2] = {64, 128};
        if ((st = encode_bf16_map(&m_dh, a->dh_in, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
      }
      CUtensorMap m_dx;
      {
        const uint64_t dims[2] = {(uint64_t)nD, (uint64_t)T};
        const uint64_t strides[1] = {(uint64_t)nD * 2};
        const uint32_t box[2] = {64, 128};
        if ((st = encode_bf16_map(&m_dx, a->dx, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
      }
      const dim3 gdx((unsigned)((T + 127) / 128), (unsigned)L.dx_slices);
      if constexpr (n % 2 == 0) {
        using Dp = tiled::DxPairCfg<n>;
        if ((st = set_smem_limit_once(tiled::dx_tc_pair_kernel<n>, Dp::SMEM))) return st;
        tiled::dx_tc_pair_kernel<n><<<gdx, tiled::kPThreads, Dp::SMEM, s>>>(
            m_x, m_dh, m_dx, img, rec, reinterpret_cast<int*>(ws), T, D, L.dx_kb_per);
      } else {
        if ((st = set_smem_limit_once(tiled::dx_tc_kernel<n>, Dc::SMEM))) return st;
        tiled::dx_tc_kernel<n><<<gdx, tiled::kGThreads, Dc::SMEM, s>>>(m_x, m_dh, m_dx, img, rec,
                                                                      reinterpret_cast<int*>(ws), T, D, L.dx_kb_per);
      }
      if ((st = after_launch())) return st;
    } else {
      float* dmT = reinterpret_cast<float*>(ws + L.dmT);
      const int64_t Tp = tiled::padded_tokens(T);
      const dim3 gtr((unsigned)(Tp / 32), (unsigned)((N + 31) / 32));
      tiled::transpose_kernel<n><<<gtr, tiled::kThreads, 0, s>>>(rec, dmT, T, Tp);
      if ((st = after_launch())) return st;
      if ((st = set_smem_limit_once(tiled::dx_kernel<n>, Dm::DX_SMEM))) return st;
      const dim3 gdx((unsigned)(Tp / tiled::kTT), (unsigned)((nD + tiled::kKT - 1) / tiled::kKT));
      tiled::dx_kernel<n><<<gdx, tiled::kThreads, Dm::DX_SMEM, s>>>(a->x, a->phi, a->gamma, rec, dmT, a->dh_in,
                                                                    a->dx, T, Tp, D);
      if ((st = after_launch())) return st;
    }
    {
      using Gc = tiled::GCfg<n>;
      CUtensorMap m_x;
      const uint64_t dims[2] = {(uint64_t)nD, (uint64_t)T};
      const uint64_t strides[1] = {(uint64_t)nD * 2};
      const uint32_t box[2] = {64, 128};
      if ((st = encode_bf16_map(&m_x, a->x, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))) return st;
      const int num_tiles = (int)((T + 127) / 128);
      uint8_t* gimg = reinterpret_cast<uint8_t*>(ws + L.gimg);
      tiled::gimg_kernel<n><<<num_tiles, 128, 0, s>>>(rec, gimg, T);
      if ((st = after_launch())) return st;
      if ((st = set_smem_limit_once(tiled::g_tc_kernel<n>, Gc::SMEM))) return st;
      const dim3 gg((unsigned)((nD + 127) / 128), (unsigned)L.P);
      tiled::g_tc_kernel<n><<<gg, tiled::kGThreads, Gc::SMEM, s>>>(m_x, gimg, gpart, reinterpret_cast<int*>(ws), nD,
                                                                   L.P, num_tiles);
      if ((st = after_launch())) return st;
    }
    generic::finalize_param_kernel<N><<<(nD + generic::kFinCols - 1) / generic::kFinCols + 3 + N, generic::kThreads, 0,
                                        s>>>(gpart, L.P, a->phi, a->gamma, a->dphi, a->dgamma, nD, abpart,
                                             (int64_t)L.rows_grid * kRowsWarps, a->dalpha, a->dbias);
    return after_launch();
  }
};

int bwd_workspace(int64_t T, int n, int D, int sms, size_t* bytes) {
  size_t b = bwd_generic_layout(T, n, D, sms).total;
  if (bwd_tc_shape(T, n, D)) b = std::max(b, bwd_tc_layout(T, D, sms).total);
  if (bwd_tiled_shape(T, n, D)) b = std::max(b, bwd_tiled_layout(T, n, D, sms).total);
  *bytes = b;
  return MHC_OK;
}

// ----------------------------------------------------------------- backward that recomputes the forward's intermediates
// mhc_bwd with inv_rms, h_mix and h_pre NULL runs the forward first (the same
// kernels as mhc_fwd, so the intermediates are the ones a forward with outflag
// would have returned, bit for bit), then the backward.  Workspace: [0,
// shared) serves the forward and then the backward (used one after the other
// on the stream, so they share their bytes and their status word), then
// inv_rms [T], h_mix [T][N], h_pre [T][n], h_post [T][n], h_res [T][n][n].
// The forward's h_in goes to the first T*D elements of dx, which the backward
// then overwrites.
struct BwdRecomputeLayout {
  size_t shared, inv_rms, h_mix, h_pre, h_post, h_res, total;
};

BwdRecomputeLayout bwd_recompute_layout(int64_t T, int n, int D, int sms) {
  BwdRecomputeLayout L{};
  size_t fw = 0, bw = 0;
  fwd_workspace(T, n, D, &fw);
  bwd_workspace(T, n, D, sms, &bw);
  const size_t N = (size_t)n * n + 2 * (size_t)n;
  size_t off = align_up(std::max(fw, bw), kWsAlign);
  L.shared = off;
  L.inv_rms = off;
  off = align_up(off + sizeof(float) * (size_t)T, kWsAlign);
  L.h_mix = off;
  off = align_up(off + sizeof(float) * (size_t)T * N, kWsAlign);
  L.h_pre = off;
  off = align_up(off + sizeof(float) * (size_t)T * n, kWsAlign);
  L.h_post = off;
  off = align_up(off + sizeof(float) * (size_t)T * n, kWsAlign);
  L.h_res = off;
  off = align_up(off + sizeof(float) * (size_t)T * n * n, kWsAlign);
  L.total = off;
  return L;
}

// ----------------------------------------------------------------- bounded-wait self test
// One thread runs, one after the other, the two bounded waits the kernels
// use, each on something that never completes: mbar_wait on an mbarrier
// nothing arrives on, and counter_wait (the fused forward's wait for another
// CTA's tile) on a global counter nothing increments.  Each gives up after
// its limit (about a second), sets the status word to MHC_ERR_DEVICE_TIMEOUT
// and the kernel returns; status[1] gets bit 0 / bit 1 for each wait that
// reported the timeout.  No fault is involved.
static __device__ int g_never_signalled = 0;

__global__ void wait_expiry_kernel(int* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_a, abort_b;
  if (threadIdx.x == 0) {
    sm100::mbar_init(sm100::smem_u32(&bar), 1);
    abort_a = 0;
    abort_b = 0;
    sm100::fence_mbarrier_init_cluster();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const sm100::WaitCtx wa{&abort_a, status};
    const bool a_done = sm100::mbar_wait(sm100::smem_u32(&bar), 0, wa);   // phase 0 never completes
    const sm100::WaitCtx wb{&abort_b, status};
    const bool b_done = sm100::counter_wait(&g_never_signalled, 1, wb);   // stays 0
    status[1] = (!a_done && abort_a ? 1 : 0) | (!b_done && abort_b ? 2 : 0);
  }
}

// ----------------------------------------------------------------- forward without a caller workspace
// Scratch of mhc_fwd_static: the forward's workspace (the status word in the
// first kWsHeaderBytes, the bf16 split-phi images, the per-tile counters)
// carved from one
// file-scope device array instead of caller memory.  Every device that loads
// the library holds the array until the process exits.
constexpr size_t kStaticScratchBytes = (size_t)16 << 20;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch in the current CUDA context.  In host
// code the symbol names a host-side shadow, so the address comes from
// cudaGetSymbolAddress, asked once per context with that context current.
// The cache is keyed by the driver's unique context id, not the device
// ordinal: after a device reset the module is loaded again into a new
// context, possibly at another address, and the old one must not be reused.
int static_scratch_address(void** out) {
  static std::mutex mu;
  static std::map<unsigned long long, void*> by_ctx;
  // Driver entry points through the runtime, so the library keeps no link-time
  // dependency on libcuda (it loads on machines without a driver).
  using GetCurrentFn = CUresult (*)(CUcontext*);
  using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrentFn get_current = reinterpret_cast<GetCurrentFn>(driver_entry_point("cuCtxGetCurrent"));
  static GetIdFn get_id = reinterpret_cast<GetIdFn>(driver_entry_point("cuCtxGetId"));
  auto current_id = [](unsigned long long* id) {
    CUcontext ctx = nullptr;
    return get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx != nullptr &&
           get_id(ctx, id) == CUDA_SUCCESS;
  };
  unsigned long long id = 0;
  const bool known_ctx = current_id(&id);
  std::lock_guard<std::mutex> g(mu);
  if (known_ctx) {
    auto it = by_ctx.find(id);
    if (it != by_ctx.end()) {
      *out = it->second;
      return MHC_OK;
    }
  }
  void* p = nullptr;
  MHC_CUDA_TRY(cudaGetSymbolAddress(&p, g_static_scratch));   // creates the primary context if none is current
  if (!p) return MHC_ERR_CUDA;
  if (!known_ctx && !current_id(&id)) return MHC_ERR_CUDA;
  by_ctx[id] = p;
  *out = p;
  return MHC_OK;
}

// ----------------------------------------------------------------- post-op
bool post_vec(const void* a, const void* b, const void* c, int D) {
  return D % 8 == 0 && aligned(a, 16) && aligned(b, 16) && aligned(c, 16);
}

template <int n>
struct PostFwd {
  static int run(const mhc_post_fwd_args* a, cudaStream_t s, int sms) {
    const int64_t T = a->tokens;
    const int D = a->D;
    const bool vec = post_vec(a->x, a->y, a->out, D);
    const int64_t runs = ((int64_t)(vec ? D / 8 : D) + 32 * post::kU - 1) / (32 * post::kU);
    const int64_t blocks =
        std::max<int64_t>(1, std::min<int64_t>((T * runs + post::kWarps - 1) / post::kWarps, (int64_t)sms * 8));
    if (vec)
      post::post_fwd_kernel<n, 8><<<(unsigned)blocks, post::kThreads, 0, s>>>(a->x, a->h_res, a->h_post, a->y, a->out,
                                                                              T, D);
    else
      post::post_fwd_kernel<n, 1><<<(unsigned)blocks, post::kThreads, 0, s>>>(a->x, a->h_res, a->h_post, a->y, a->out,
                                                                              T, D);
    return after_launch();
  }
};

template <int n>
struct PostBwd {
  static int run(const mhc_post_bwd_args* a, cudaStream_t s, int sms) {
    const int64_t T = a->tokens;
    const int D = a->D;
    const bool vec = post_vec(a->x, a->y, a->dout, D) && aligned(a->dx, 16) && aligned(a->dy, 16);
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((T + post::kWarps - 1) / post::kWarps,
                                                                  (int64_t)sms * 8));
    if (vec)
      post::post_bwd_kernel<n, 8><<<(unsigned)blocks, post::kThreads, 0, s>>>(
          a->x, a->h_res, a->h_post, a->y, a->dout, a->dx, a->dy, a->dh_res, a->dh_post, T, D);
    else
      post::post_bwd_kernel<n, 1><<<(unsigned)blocks, post::kThreads, 0, s>>>(
          a->x, a->h_res, a->h_post, a->y, a->dout, a->dx, a->dy, a->dh_res, a->dh_post, T, D);
    return after_launch();
  }
};

// The plan of mhc_query_plan / mhc_query_plan_for (shape already checked).
int query_plan_impl(int which, int64_t tokens, int n, int D, int sms, bool fused_ok, int* path, int* cluster_size,
                    int* clusters) {
  *path = 0;
  *cluster_size = 0;
  *clusters = 0;
  if (which == 0 && fwd_tc_shape(tokens, n, D)) {
    const FwdTcPlan fp = fwd_tc_plan_with(tokens, n, D, sms, fused_ok);
    *path = fp.fused ? 2 : 1;
    *cluster_size = fp.S_K;
    *clusters = fp.grid;
  } else if (which == 1 && bwd_tc_shape(tokens, n, D)) {
    const BwdTcPlan bp = bwd_tc_plan(tokens, D, sms);
    *path = 1;
    *cluster_size = bp.S_K;
    *clusters = bp.S_T;
  } else if (which == 1 && bwd_tiled_shape(tokens, n, D)) {
    const BwdTiledLayout L = bwd_tiled_layout(tokens, n, D, sms);
    *path = 3;
    *cluster_size = L.P;
    *clusters = L.dx_tc ? (L.dx_pair ? 2 : 1) : 0;
  } else if (which != 0 && which != 1) {
    return MHC_ERR_BAD_SHAPE;
  }
  return MHC_OK;
}

}  // namespace
}  // namespace mhc

using namespace mhc;

extern "C" {

const char* mhc_status_string(int status) {
  switch (status) {
    case MHC_OK: return "ok";
    case MHC_ERR_NULL_POINTER: return "a required pointer is NULL";
    case MHC_ERR_BAD_SHAPE: return "unsupported shape (need T >= 0, 1 <= n <= 8, D >= 1)";
    case MHC_ERR_MISALIGNED: return "a pointer is not aligned to its element size";
    case MHC_ERR_WORKSPACE_TOO_SMALL: return "workspace smaller than the *_workspace_size answer";
    case MHC_ERR_CUDA: return "a CUDA call failed";
    case MHC_ERR_DEVICE_TIMEOUT: return "a kernel's bounded wait expired";
    case MHC_ERR_NO_DEVICE: return "the current device is not an sm_100 GPU";
    case MHC_ERR_LIMIT: return "a size is beyond this entry point's fixed limit";
    case MHC_ERR_OUT_OF_BOUNDS: return "a debug-bounds build saw an access outside the call's buffers";
    case MHC_ERR_UNSUPPORTED: return "the entry point is not compiled into this library";
    default: return "unknown mhc status";
  }
}

const char* mhc_last_cuda_error(void) { return t_last_cuda_error.c_str(); }

int mhc_abi_version(void) { return 10400; }

uint64_t mhc_launch_count(void) { return g_launch_count.load(std::memory_order_relaxed); }

int mhc_fwd_workspace_size(int64_t tokens, int32_t n, int32_t D, size_t* bytes) {
  if (!bytes) return MHC_ERR_NULL_POINTER;
  int st = check_shape(tokens, n, D);
  if (st) return st;
  return fwd_workspace(tokens, n, D, bytes);
}

int mhc_bwd_workspace_size(int64_t tokens, int32_t n, int32_t D, size_t* bytes) {
  if (!bytes) return MHC_ERR_NULL_POINTER;
  int st = check_shape(tokens, n, D);
  if (st) return st;
  int sms = 0;
  if ((st = current_sm_count(&sms))) return st;
  return bwd_workspace(tokens, n, D, sms, bytes);
}

}  // extern "C"

namespace mhc {
namespace {
// Debug-bounds builds: the buffers of the current call, copied to the
// device's table in stream order before its kernels (common.cuh).  Absent
// from normal builds.
#ifdef MHC_DEBUG_BOUNDS
struct DbgTable {
  DbgBuf b[kDbgBufs];
  int n = 0;
  void add(const void* p, size_t bytes) {
    if (!p || bytes == 0 || n >= kDbgBufs) return;
    const unsigned long long lo = reinterpret_cast<unsigned long long>(p);
    b[n++] = DbgBuf{lo, lo + bytes};
  }
  // the source is pageable host memory: the copy has taken it when the call returns
  int upload(cudaStream_t s) const {
    MHC_CUDA_TRY(cudaMemcpyToSymbolAsync(g_dbg_bufs, b, sizeof(DbgBuf) * kDbgBufs, 0, cudaMemcpyHostToDevice, s));
    MHC_CUDA_TRY(cudaMemcpyToSymbolAsync(g_dbg_nbufs, &n, sizeof(int), 0, cudaMemcpyHostToDevice, s));
    return MHC_OK;
  }
};

int dbg_register_fwd(const mhc_fwd_args* a, const FwdEx& ex, cudaStream_t s) {
  const size_t T = (size_t)a->tokens, n = (size_t)a->n, D = (size_t)a->D, N = n * n + 2 * n;
  DbgTable t;
  t.add(a->x, T * n * D * 2);
  t.add(ex.x_fp8, T * n * D);
  t.add(ex.x_exp, T);
  t.add(a->phi, N * n * D * 4);
  t.add(ex.phi_bf16, N * n * D * 2);
  t.add(a->alpha, 3 * 4);
  t.add(a->bias, N * 4);
  t.add(a->h_in, T * D * 2);
  t.add(a->h_post, T * n * 4);
  t.add(a->h_res, T * n * n * 4);
  t.add(a->inv_rms, T * 4);
  t.add(a->h_mix, T * N * 4);
  t.add(a->h_pre, T * n * 4);
  t.add(ex.h_in_rstd, T * 4);
  t.add(a->workspace, a->workspace_bytes);
  return t.upload(s);
}

int dbg_register_bwd(const mhc_bwd_args* a, cudaStream_t s) {
  const size_t T = (size_t)a->tokens, n = (size_t)a->n, D = (size_t)a->D, N = n * n + 2 * n;
  DbgTable t;
  t.add(a->x, T * n * D * 2);
  t.add(a->phi, N * n * D * 4);
  t.add(a->alpha, 3 * 4);
  t.add(a->bias, N * 4);
  t.add(a->inv_rms, T * 4);
  t.add(a->h_mix, T * N * 4);
  t.add(a->h_pre, T * n * 4);
  t.add(a->h_post, T * n * 4);
  t.add(a->dh_in, T * D * 2);
  t.add(a->dh_post, T * n * 4);
  t.add(a->dh_res, T * n * n * 4);
  t.add(a->gamma, n * D * 4);
  t.add(a->dx, T * n * D * 2);
  t.add(a->dphi, N * n * D * 4);
  t.add(a->dalpha, 3 * 4);
  t.add(a->dbias, N * 4);
  t.add(a->dgamma, n * D * 4);
  t.add(a->workspace, a->workspace_bytes);
  return t.upload(s);
}

template <class A>
int dbg_register_post(const A* a, const void* const* ptrs, const size_t* sizes, int count, cudaStream_t s) {
  (void)a;
  DbgTable t;
  for (int i = 0; i < count; ++i) t.add(ptrs[i], sizes[i]);
  return t.upload(s);
}

__global__ void dbg_selftest_kernel(const char* buf) {
  // one byte past the registered 256 bytes: the check fails, nothing is read
  (void)MHC_CHK(buf + 256, 1);
}
#endif

// mhc_fwd and mhc_fwd_ex: validation, then fwd_run.
int fwd_entry(const mhc_fwd_args* a, const FwdEx& ex, void* stream) {
  if (!a) return MHC_ERR_NULL_POINTER;
  int st = check_shape(a->tokens, a->n, a->D);
  if (st) return st;
  if (!a->workspace) return MHC_ERR_NULL_POINTER;
  const bool bf16_phi = ex.phi_bf16 != nullptr;
  size_t need = 0;
  fwd_workspace(a->tokens, a->n, a->D, &need, bf16_phi);
  if (a->workspace_bytes < need) return MHC_ERR_WORKSPACE_TOO_SMALL;
  if (!aligned(a->workspace, kWsAlign)) return MHC_ERR_MISALIGNED;
  int sms = 0;
  if ((st = current_sm_count(&sms))) return st;
  if (ex.sm_budget < 0) return MHC_ERR_BAD_SHAPE;
  if (ex.sm_budget > 0) sms = std::min(sms, ex.sm_budget);
  if (a->tokens == 0) return MHC_OK;
  if ((!a->x && !ex.x_fp8) || (!a->phi && !bf16_phi) || !a->alpha || !a->bias || !a->h_in || !a->h_post ||
      !a->h_res)
    return MHC_ERR_NULL_POINTER;
  if (ex.x_fp8 && !((a->n == 4 || a->n == 8) && fwd_tc_shape(a->tokens, a->n, a->D) && aligned(ex.x_fp8, 16) &&
                    aligned(a->h_in, 16)))
    return MHC_ERR_BAD_SHAPE;
  if (!aligned(a->x, 2) || !aligned(a->h_in, 2) || !aligned(a->phi, 4) || !aligned(a->alpha, 4) ||
      !aligned(a->bias, 4) || !aligned(a->h_post, 4) || !aligned(a->h_res, 4) || !aligned(a->inv_rms, 4) ||
      !aligned(a->h_mix, 4) || !aligned(a->h_pre, 4) || !aligned(ex.phi_bf16, 2) || !aligned(ex.h_in_rstd, 4))
    return MHC_ERR_MISALIGNED;
#ifdef MHC_DEBUG_BOUNDS
  if ((st = dbg_register_fwd(a, ex, static_cast<cudaStream_t>(stream)))) return st;
#endif
  return fwd_run(a, ex, static_cast<cudaStream_t>(stream), sms);
}
}  // namespace
}  // namespace mhc

extern "C" {

int mhc_fwd(const mhc_fwd_args* a, void* stream) { return fwd_entry(a, FwdEx{}, stream); }

int mhc_fwd_ex_workspace_size(const mhc_fwd_ex_args* ex, int64_t tokens, int32_t n, int32_t D, size_t* bytes) {
  if (!bytes) return MHC_ERR_NULL_POINTER;
  int st = check_shape(tokens, n, D);
  if (st) return st;
  return fwd_workspace(tokens, n, D, bytes, ex != nullptr && ex->phi_bf16 != nullptr);
}

int mhc_fwd_ex(const mhc_fwd_args* a, const mhc_fwd_ex_args* ex, void* stream) {
  FwdEx e;
  if (ex) {
    e.phi_bf16 = ex->phi_bf16;
    e.h_in_rstd = ex->h_in_rstd;
    e.h_in_eps = ex->h_in_eps;
    e.sm_budget = ex->sm_budget;
    e.x_fp8 = ex->x_fp8;
    e.x_exp = ex->x_exp;
  }
  return fwd_entry(a, e, stream);
}

int mhc_bwd(const mhc_bwd_args* a, void* stream) {
  if (!a) return MHC_ERR_NULL_POINTER;
  int st = check_shape(a->tokens, a->n, a->D);
  if (st) return st;
  if (!a->workspace) return MHC_ERR_NULL_POINTER;
  int sms = 0;
  if ((st = current_sm_count(&sms))) return st;
  const bool recompute = !a->inv_rms && !a->h_mix && !a->h_pre;
  size_t need = 0;
  if (recompute) need = bwd_recompute_layout(a->tokens, a->n, a->D, sms).total;
  else if ((st = bwd_workspace(a->tokens, a->n, a->D, sms, &need))) return st;
  if (a->workspace_bytes < need) return MHC_ERR_WORKSPACE_TOO_SMALL;
  if (!aligned(a->workspace, kWsAlign)) return MHC_ERR_MISALIGNED;
  if (!a->dphi || !a->dalpha || !a->dbias || !a->dgamma || !a->alpha || !a->phi) return MHC_ERR_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int N = a->n * a->n + 2 * a->n;
  if (a->tokens == 0) {
    MHC_CUDA_TRY(cudaMemsetAsync(a->dphi, 0, sizeof(float) * (size_t)N * a->n * a->D, s));
    MHC_CUDA_TRY(cudaMemsetAsync(a->dgamma, 0, sizeof(float) * (size_t)a->n * a->D, s));
    MHC_CUDA_TRY(cudaMemsetAsync(a->dalpha, 0, sizeof(float) * 3, s));
    MHC_CUDA_TRY(cudaMemsetAsync(a->dbias, 0, sizeof(float) * (size_t)N, s));
    return MHC_OK;
  }
  if (recompute) {
    // the forward into the workspace, then the backward from its intermediates
    if (!a->x || !a->bias || !a->dx) return MHC_ERR_NULL_POINTER;
    const BwdRecomputeLayout L = bwd_recompute_layout(a->tokens, a->n, a->D, sms);
    char* ws = static_cast<char*>(a->workspace);
    mhc_fwd_args f{};
    f.x = a->x;
    f.phi = a->phi;
    f.alpha = a->alpha;
    f.bias = a->bias;
    f.h_in = a->dx;
    f.h_post = reinterpret_cast<float*>(ws + L.h_post);
    f.h_res = reinterpret_cast<float*>(ws + L.h_res);
    f.inv_rms = reinterpret_cast<float*>(ws + L.inv_rms);
    f.h_mix = reinterpret_cast<float*>(ws + L.h_mix);
    f.h_pre = reinterpret_cast<float*>(ws + L.h_pre);
    f.tokens = a->tokens;
    f.n = a->n;
    f.D = a->D;
    f.norm_eps = a->norm_eps;
    f.hc_eps = a->hc_eps;
    f.workspace = a->workspace;
    f.workspace_bytes = L.shared;
    if ((st = mhc_fwd(&f, stream))) return st;
    mhc_bwd_args b = *a;
    b.inv_rms = f.inv_rms;
    b.h_mix = f.h_mix;
    b.h_pre = f.h_pre;
    if (!b.h_post) b.h_post = f.h_post;
    b.workspace_bytes = L.shared;
    return mhc_bwd(&b, stream);
  }
  if (!a->x || !a->inv_rms || !a->h_mix || !a->h_pre || !a->h_post || !a->dh_in || !a->dh_post ||
      !a->dh_res || !a->dx)
    return MHC_ERR_NULL_POINTER;
  if (!aligned(a->x, 2) || !aligned(a->dh_in, 2) || !aligned(a->dx, 2) || !aligned(a->phi, 4) ||
      !aligned(a->inv_rms, 4) || !aligned(a->h_mix, 4) || !aligned(a->h_pre, 4) || !aligned(a->h_post, 4) ||
      !aligned(a->dh_post, 4) || !aligned(a->dh_res, 4) || !aligned(a->gamma, 4) || !aligned(a->dphi, 4) ||
      !aligned(a->dalpha, 4) || !aligned(a->dbias, 4) || !aligned(a->dgamma, 4))
    return MHC_ERR_MISALIGNED;
#ifdef MHC_DEBUG_BOUNDS
  if ((st = dbg_register_bwd(a, s))) return st;
#endif
  if (bwd_tc_eligible(a)) return bwd_tc_run(a, s, sms);
  if (bwd_tiled_eligible(a)) return dispatch_n<BwdTiled>(a->n, a, s, sms);
  return dispatch_n<BwdGeneric>(a->n, a, s, sms);
}

int mhc_fwd_static(const mhc_fwd_args* a, void* stream) {
  if (!a) return MHC_ERR_NULL_POINTER;
  int st = check_shape(a->tokens, a->n, a->D);
  if (st) return st;
  size_t need = 0;
  fwd_workspace(a->tokens, a->n, a->D, &need);
  if (need > kStaticScratchBytes) return MHC_ERR_LIMIT;
  int sms = 0;
  if ((st = current_sm_count(&sms))) return st;
  void* scratch = nullptr;
  if ((st = static_scratch_address(&scratch))) return st;
  // Same validation and kernels as mhc_fwd; only the workspace differs.  The
  // split-phi images are rewritten in full (padding rows included) and the
  // tile counters zeroed by every call, and the status word is only ever
  // written, so nothing in the array has to start at zero.
  mhc_fwd_args b = *a;
  b.workspace = scratch;
  b.workspace_bytes = kStaticScratchBytes;
  return mhc_fwd(&b, stream);
}

int mhc_selftest_wait_expiry(void* workspace, void* stream) {
  if (!workspace) return MHC_ERR_NULL_POINTER;
  if (!aligned(workspace, kWsAlign)) return MHC_ERR_MISALIGNED;
  int sms = 0;
  int st = current_sm_count(&sms);
  if (st) return st;
  wait_expiry_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<int*>(workspace));
  return after_launch();
}

int mhc_query_plan(int which, int64_t tokens, int32_t n, int32_t D, int* path, int* cluster_size, int* clusters) {
  if (!path || !cluster_size || !clusters) return MHC_ERR_NULL_POINTER;
  int st = check_shape(tokens, n, D);
  if (st) return st;
  int sms = 0;
  if ((st = current_sm_count(&sms))) return st;
  const bool fused_ok = which == 0 && n == 4 && fwd_fused_supported(n);
  return query_plan_impl(which, tokens, n, D, sms, fused_ok, path, cluster_size, clusters);
}

int mhc_query_plan_for(int which, int64_t tokens, int32_t n, int32_t D, int32_t sms, int* path, int* cluster_size,
                       int* clusters) {
  if (!path || !cluster_size || !clusters) return MHC_ERR_NULL_POINTER;
  int st = check_shape(tokens, n, D);
  if (st) return st;
  if (sms < 1 || sms > 4096) return MHC_ERR_BAD_SHAPE;
  return query_plan_impl(which, tokens, n, D, sms, n == 4, path, cluster_size, clusters);
}

int mhc_bwd_recompute_workspace_size(int64_t tokens, int32_t n, int32_t D, size_t* bytes) {
  if (!bytes) return MHC_ERR_NULL_POINTER;
  int st = check_shape(tokens, n, D);
  if (st) return st;
  int sms = 0;
  if ((st = current_sm_count(&sms))) return st;
  *bytes = bwd_recompute_layout(tokens, n, D, sms).total;
  return MHC_OK;
}

int mhc_query_bwd_grid(int64_t tokens, int32_t n, int32_t D, int32_t sms, int32_t* grid) {
  if (!grid) return MHC_ERR_NULL_POINTER;
  int st = check_shape(tokens, n, D);
  if (st) return st;
  if (sms < 0 || sms > 4096) return MHC_ERR_BAD_SHAPE;
  if (sms == 0 && (st = current_sm_count(&sms))) return st;
  if (!bwd_tc_shape(tokens, n, D)) return MHC_ERR_BAD_SHAPE;
  const BwdTcPlan p = bwd_tc_plan(tokens, D, sms);
  const int32_t v[6] = {p.Dc, p.S_K, p.S_T, p.J, p.E, p.R};
  for (int i = 0; i < 6; ++i) grid[i] = v[i];
  return MHC_OK;
}

int mhc_bwd_workspace_size_for(int64_t tokens, int32_t n, int32_t D, int32_t sms, size_t* bytes) {
  if (!bytes) return MHC_ERR_NULL_POINTER;
  int st = check_shape(tokens, n, D);
  if (st) return st;
  if (sms < 1 || sms > 4096) return MHC_ERR_BAD_SHAPE;
  return bwd_workspace(tokens, n, D, sms, bytes);
}

int mhc_post_fwd(const mhc_post_fwd_args* a, void* stream) {

  if (!a) return MHC_ERR_NULL_POINTER;
  int st = check_shape(a->tokens, a->n, a->D);
  if (st) return st;
  int sms = 0;
  if ((st = current_sm_count(&sms))) return st;
  if (a->tokens == 0) return MHC_OK;
  if (!a->x || !a->h_res || !a->h_post || !a->y || !a->out) return MHC_ERR_NULL_POINTER;
  if (!aligned(a->x, 2) || !aligned(a->y, 2) || !aligned(a->out, 2) || !aligned(a->h_res, 4) ||
      !aligned(a->h_post, 4))
    return MHC_ERR_MISALIGNED;
#ifdef MHC_DEBUG_BOUNDS
  {
    const size_t T = (size_t)a->tokens, n = (size_t)a->n, D = (size_t)a->D;
    const void* ptrs[5] = {a->x, a->h_res, a->h_post, a->y, a->out};
    const size_t sizes[5] = {T * n * D * 2, T * n * n * 4, T * n * 4, T * D * 2, T * n * D * 2};
    if ((st = dbg_register_post(a, ptrs, sizes, 5, static_cast<cudaStream_t>(stream)))) return st;
  }
#endif
  return dispatch_n<PostFwd>(a->n, a, static_cast<cudaStream_t>(stream), sms);
}

int mhc_post_bwd(const mhc_post_bwd_args* a, void* stream) {
  if (!a) return MHC_ERR_NULL_POINTER;
  int st = check_shape(a->tokens, a->n, a->D);
  if (st) return st;
  int sms = 0;
  if ((st = current_sm_count(&sms))) return st;
  if (a->tokens == 0) return MHC_OK;
  if (!a->x || !a->h_res || !a->h_post || !a->y || !a->dout || !a->dx || !a->dy || !a->dh_res || !a->dh_post)
    return MHC_ERR_NULL_POINTER;
  if (!aligned(a->x, 2) || !aligned(a->y, 2) || !aligned(a->dout, 2) || !aligned(a->dx, 2) ||
      !aligned(a->dy, 2) || !aligned(a->h_res, 4) || !aligned(a->h_post, 4) || !aligned(a->dh_res, 4) ||
      !aligned(a->dh_post, 4))
    return MHC_ERR_MISALIGNED;
#ifdef MHC_DEBUG_BOUNDS
  {
    const size_t T = (size_t)a->tokens, n = (size_t)a->n, D = (size_t)a->D;
    const void* ptrs[9] = {a->x, a->h_res, a->h_post, a->y, a->dout, a->dx, a->dy, a->dh_res, a->dh_post};
    const size_t sizes[9] = {T * n * D * 2, T * n * n * 4, T * n * 4, T * D * 2, T * n * D * 2,
                             T * n * D * 2, T * D * 2,     T * n * n * 4, T * n * 4};
    if ((st = dbg_register_post(a, ptrs, sizes, 9, static_cast<cudaStream_t>(stream)))) return st;
  }
#endif
  return dispatch_n<PostBwd>(a->n, a, static_cast<cudaStream_t>(stream), sms);
}

int mhc_debug_bounds(uint64_t* record, int clear) {
  if (!record) return MHC_ERR_NULL_POINTER;
  for (int i = 0; i < 4; ++i) record[i] = 0;
#ifdef MHC_DEBUG_BOUNDS
  MHC_CUDA_TRY(cudaDeviceSynchronize());
  unsigned long long r[4] = {0, 0, 0, 0};
  MHC_CUDA_TRY(cudaMemcpyFromSymbol(r, g_dbg_oob, sizeof(r)));
  if (clear) {
    const unsigned long long z[4] = {0, 0, 0, 0};
    MHC_CUDA_TRY(cudaMemcpyToSymbol(g_dbg_oob, z, sizeof(z)));
  }
  for (int i = 0; i < 4; ++i) record[i] = r[i];
  return r[0] == 0 ? MHC_OK : MHC_ERR_OUT_OF_BOUNDS;
#else
  (void)clear;
  return MHC_ERR_UNSUPPORTED;
#endif
}

int mhc_debug_bounds_selftest(void* workspace, void* stream) {
#ifdef MHC_DEBUG_BOUNDS
  if (!workspace) return MHC_ERR_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DbgTable t;
  t.add(workspace, 256);
  int st;
  if ((st = t.upload(s))) return st;
  dbg_selftest_kernel<<<1, 1, 0, s>>>(static_cast<const char*>(workspace));
  return after_launch();
#else
  (void)workspace;
  (void)stream;
  return MHC_ERR_UNSUPPORTED;
#endif
}

int mhc_read_device_status(void* workspace, void* stream, int* device_status) {
  if (!workspace || !device_status) return MHC_ERR_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host = 0;
  MHC_CUDA_TRY(cudaMemcpyAsync(&host, workspace, sizeof(int), cudaMemcpyDeviceToHost, s));
  MHC_CUDA_TRY(cudaStreamSynchronize(s));
  MHC_CUDA_TRY(cudaMemsetAsync(workspace, 0, sizeof(int), s));
  MHC_CUDA_TRY(cudaStreamSynchronize(s));
  *device_status = host;
  return MHC_OK;
}

}  // extern "C"
