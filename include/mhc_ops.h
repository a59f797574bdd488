/*
 * mhc_ops.h -- C ABI of the B200 (sm_100a) mHC pre-op library (libmhc_ops.so).
 *
 * The manifold-constrained hyper-connection pre-op of folrent1896/mhc_ops,
 * forward and backward.  Every entry point takes plain device pointers and
 * sizes, launches on the given CUDA stream (a cudaStream_t passed as void*;
 * NULL = legacy default stream) and returns an mhc_status.  No entry point
 * allocates device memory except where its comment says so: scratch comes
 * from a caller-owned workspace whose size the *_workspace_size query returns.
 * Calls hold no global mutable state and may be issued from several host
 * threads; two calls that share one workspace must be ordered on the device.
 * A workspace must be zero-filled once before its first use (its first
 * bytes hold the device status word, see mhc_read_device_status).
 *
 * Shapes: T tokens (= B*S of the reference), n streams, D hidden, nD = n*D,
 * N = n*n + 2n.  Tensors are dense row-major:
 *   x [T,n,D] bf16, phi [N,nD] f32, alpha [3] f32, bias [N] f32,
 *   h_in [T,D] bf16, h_post [T,n] f32, h_res [T,n,n] f32,
 *   inv_rms [T] f32, h_mix [T,N] f32 (pre-RMS projection), h_pre [T,n] f32,
 *   dh_in [T,D] bf16, dh_post [T,n] f32, dh_res [T,n,n] f32, gamma [n,D] f32,
 *   dx [T,n,D] bf16, dphi [N,nD] f32, dalpha [3] f32, dbias [N] f32,
 *   dgamma [nD] f32 (flat, as the reference golden returns it).
 * bf16 values are passed as uint16_t bit patterns.
 * Supported: 1 <= n <= 8, D >= 1, T >= 0; pointers 16-byte aligned and
 * D a multiple of 8 for the tensor-core kernels (other shapes run the
 * generic CUDA kernels).
 */
#ifndef MHC_OPS_H_
#define MHC_OPS_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MHC_API __attribute__((visibility("default")))
#else
#define MHC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum mhc_status {
  MHC_OK = 0,
  MHC_ERR_NULL_POINTER = 1,        /* a required pointer is NULL */
  MHC_ERR_BAD_SHAPE = 2,           /* T < 0, n outside [1,8], D < 1, or overflow */
  MHC_ERR_MISALIGNED = 3,          /* a pointer is not 16-byte aligned */
  MHC_ERR_WORKSPACE_TOO_SMALL = 4, /* workspace_bytes below the *_workspace_size answer */
  MHC_ERR_CUDA = 5,                /* a CUDA runtime/driver call failed (see mhc_last_cuda_error) */
  MHC_ERR_DEVICE_TIMEOUT = 6,      /* a kernel's bounded wait expired (read by mhc_read_device_status) */
  MHC_ERR_NO_DEVICE = 7,           /* no sm_100 device is current */
  MHC_ERR_LIMIT = 8,               /* a size beyond a fixed limit of the entry point */
  MHC_ERR_OUT_OF_BOUNDS = 9,       /* a debug-bounds build saw an access outside the call's buffers */
  MHC_ERR_UNSUPPORTED = 10         /* the entry point is not compiled into this library */
} mhc_status;

/* Forward arguments.  Replaces the Python signature
 *   mhc_forward_pre(x, phi, alpha, bias, outflag=False, norm_eps=1e-6, hc_eps=1e-6)
 * of the reference (src/forward/golden.py:10-11; Triton twin
 * src/forward/mhc_forward_pre_triton.py:409-417).  inv_rms, h_mix and h_pre
 * are the outflag outputs (golden.py:65-69): pass NULL to skip writing them. */
typedef struct mhc_fwd_args {
  const uint16_t* x;
  const float* phi;
  const float* alpha;
  const float* bias;
  uint16_t* h_in;
  float* h_post;
  float* h_res;
  float* inv_rms;   /* optional */
  float* h_mix;     /* optional */
  float* h_pre;     /* optional */
  int64_t tokens;
  int32_t n;
  int32_t D;
  float norm_eps;
  float hc_eps;
  void* workspace;
  size_t workspace_bytes;
} mhc_fwd_args;

/* Backward arguments.  Replaces the Python signature
 *   mhc_backward_manual(x, phi, alpha, bias, inv_rms, h_mix, h_pre, h_post,
 *                       dh_in, dh_post, dh_res, gamma, norm_eps=1e-6, hc_eps=1e-6)
 * of the reference (src/backward/golden.py:10-13, returns at :96; Triton twin
 * src/backward/mhc_backward_triton.py:467-473).  gamma may be NULL (all ones).
 * bias and norm_eps are unused by the math, as in the reference, except in
 * the recompute form: with inv_rms, h_mix and h_pre all NULL, mhc_bwd first
 * runs the forward (the kernels of mhc_fwd, with these phi, alpha, bias and
 * eps) to recompute them -- a forward that did not store its outflag outputs
 * (116 bytes per token at n = 4) pays one more read of x and the projection
 * instead -- and h_post may then be NULL as well.  The recomputed values are
 * bit for bit those mhc_fwd returns, so the results equal the stored form's.
 * That form needs mhc_bwd_recompute_workspace_size bytes of workspace and
 * uses dx as scratch before writing it.  (The reference contract returns
 * the intermediates from the forward, src/forward/golden.py:65-69.) */
typedef struct mhc_bwd_args {
  const uint16_t* x;
  const float* phi;
  const float* alpha;
  const float* bias;     /* read by the recompute form only; else may be NULL */
  const float* inv_rms;
  const float* h_mix;
  const float* h_pre;
  const float* h_post;
  const uint16_t* dh_in;
  const float* dh_post;
  const float* dh_res;
  const float* gamma;    /* optional */
  uint16_t* dx;
  float* dphi;
  float* dalpha;
  float* dbias;
  float* dgamma;
  int64_t tokens;
  int32_t n;
  int32_t D;
  float norm_eps;
  float hc_eps;
  void* workspace;
  size_t workspace_bytes;
} mhc_bwd_args;

/* Human-readable text for a status code (static storage). */
MHC_API const char* mhc_status_string(int status);

/* Text of the last CUDA error seen by this thread inside the library. */
MHC_API const char* mhc_last_cuda_error(void);

/* Workspace bytes mhc_fwd needs for this shape on the current device.
 * Replaces nothing in the reference (its wrappers allocate with torch.empty,
 * src/forward/mhc_forward_pre_triton.py:437,466). */
MHC_API int mhc_fwd_workspace_size(int64_t tokens, int32_t n, int32_t D, size_t* bytes);

/* Forward pass; see mhc_fwd_args.  Replaces mhc_forward_pre
 * (src/forward/golden.py:10-69) and mhc_forward_pre_triton_optimized
 * (src/forward/mhc_forward_pre_triton.py:409-514). */
MHC_API int mhc_fwd(const mhc_fwd_args* args, void* stream);

/* Forward pass that allocates nothing and takes no workspace: for callers that
 * may not call cudaMalloc, such as a host whose allocator owns all device
 * memory or a runtime that plans memory ahead and forbids allocation in its
 * serving loop.  No counterpart in the reference.
 *
 * Same arguments, validation, kernels and results as mhc_fwd, except that
 * args->workspace and args->workspace_bytes are ignored.  The scratch the
 * forward needs (the bf16 split-phi images, 160 bytes per element of phi's
 * n*D row for n = 4 and 320 for n = 8, plus 4 bytes per 128 tokens) comes
 * from one 16 MiB device array inside the library.  Every GPU that loads the
 * library holds those 16 MiB until the process exits.
 *   Limit: a shape needing more than 16 MiB returns MHC_ERR_LIMIT.  Up to
 *   778,240 tokens that means D > 26176 for n = 4 and D > 6528 for n = 8
 *   (D a multiple of 64); more tokens lower the limit by 4 bytes per 128
 *   tokens.  Other shapes need only the 256-byte status header.
 *   The first call in each CUDA context (one per device; a new one after a
 *   device reset) looks up the array's device address in that context.  Make
 *   that first call before any stream capture.
 *   Every call on a device uses the same array.  Calls that overlap on the
 *   GPU (two streams, or two host threads) race on it and may return wrong
 *   results.  Order them on one stream, or use mhc_fwd with a workspace per
 *   stream.  The array keeps the previous call's contents.  Nothing in it
 *   must start at zero, because each call rewrites all the scratch it reads.
 *   A bounded-wait timeout sets the array's status word, which no entry
 *   point returns.  Use mhc_fwd and mhc_read_device_status when you need it. */
MHC_API int mhc_fwd_static(const mhc_fwd_args* args, void* stream);

/* Options of mhc_fwd_ex.  Each is off when its pointer is NULL.
 *   phi_bf16: phi given as bf16 bit patterns [N, nD] instead of fp32
 *     (args->phi is then ignored and may be NULL).  A bf16 phi is exact in
 *     one bf16 term, so the projection runs one tensor-core product per
 *     K-step instead of the three (n <= 5) or two of an fp32 phi.
 *   h_in_rstd: [T] f32 output, 1 / sqrt(mean_d(h_in[t,d]^2) + h_in_eps) over
 *     the bf16 h_in row: the factor of the RMSNorm that opens the next
 *     sublayer, computed while h_in is written, so that sublayer need not
 *     read h_in once more to reduce it.
 *   sm_budget: when > 0, the most SMs the forward's grids occupy.  The
 *     fused forward is one cooperative launch with a CTA on every SM, so a
 *     collective still running on a few SMs (a data-parallel all-reduce of
 *     the previous step's gradients) would hold it back until it ends; with
 *     the SMs that collective uses left out, the two run side by side.
 *   x_fp8, x_exp: x given as e4m3 bytes [T, n, D] (args->x is then ignored
 *     and may be NULL) with a power-of-two scale per token:
 *     x[t,:] = x_fp8[t,:] * 2^x_exp[t] (x_exp may be NULL: exponent 0).
 *     Every such value is exact in bf16, and the outputs are bit for bit
 *     those of mhc_fwd on that bf16 x; the forward reads half the bytes of
 *     x.  For inference (the backward takes bf16 x).  Tensor-core shapes
 *     only (n in {4, 8}, D a multiple of 64, x_fp8 16-byte aligned; others
 *     return MHC_ERR_BAD_SHAPE); keep x * 2^e inside the bf16 range. 
 * No counterpart in the reference (its forward takes bf16 x and fp32 phi and
 * stops at h_in, src/forward/golden.py:38,41,62-63). */
typedef struct mhc_fwd_ex_args {
  const uint16_t* phi_bf16;
  float* h_in_rstd;
  float h_in_eps;
  int32_t sm_budget;
  const uint8_t* x_fp8;
  const int8_t* x_exp;
} mhc_fwd_ex_args;
/* Workspace bytes mhc_fwd_ex needs with these options (ex may be NULL). */
MHC_API int mhc_fwd_ex_workspace_size(const mhc_fwd_ex_args* ex, int64_t tokens, int32_t n, int32_t D,
                                      size_t* bytes);
/* mhc_fwd with the options above (ex may be NULL: then exactly mhc_fwd). */
MHC_API int mhc_fwd_ex(const mhc_fwd_args* args, const mhc_fwd_ex_args* ex, void* stream);
/* Workspace bytes mhc_bwd needs for this shape on the current device.
 * Replaces the intermediates the Triton backward allocates
 * (src/backward/mhc_backward_triton.py:509-510). */
MHC_API int mhc_bwd_workspace_size(int64_t tokens, int32_t n, int32_t D, size_t* bytes);

/* Backward pass; see mhc_bwd_args.  Replaces mhc_backward_manual
 * (src/backward/golden.py:10-96) and mhc_backward_triton
 * (src/backward/mhc_backward_triton.py:467-729).  The parameter gradients
 * dphi, dgamma, dalpha, dbias are reduced over tokens in a fixed order, so
 * repeated calls return identical bytes. */
MHC_API int mhc_bwd(const mhc_bwd_args* args, void* stream);

/* Workspace bytes mhc_bwd needs when it recomputes the forward's
 * intermediates (inv_rms, h_mix and h_pre all NULL), on the current device. */
MHC_API int mhc_bwd_recompute_workspace_size(int64_t tokens, int32_t n, int32_t D, size_t* bytes);
/* Reads (and clears) the device status word a previous mhc_fwd / mhc_bwd
 * left in `workspace`; synchronizes `stream`.  *device_status receives
 * MHC_OK or MHC_ERR_DEVICE_TIMEOUT.  No counterpart in the reference, which
 * has no bounded device waits. */
MHC_API int mhc_read_device_status(void* workspace, void* stream, int* device_status);

/* Self test of the device-side failure detection: launches one CTA that
 * runs the two bounded waits the tensor-core kernels use, each on something
 * that never completes (an mbarrier nothing arrives on; a global counter
 * nothing increments, as the fused forward waits on other CTAs' tiles).
 * Each wait gives up after about a second; the kernel writes
 * MHC_ERR_DEVICE_TIMEOUT into the workspace's status word (read it with
 * mhc_read_device_status), sets bits 0 and 1 of the second int of the
 * workspace for the two waits that reported it, and returns; the context
 * stays usable.  No counterpart in the reference (it has no device waits). */
MHC_API int mhc_selftest_wait_expiry(void* workspace, void* stream);

/* Launch plan the library uses for this shape on the current device:
 * *path = 0 generic kernels, 1 tensor-core kernels, 2 (forward only) the
 * fused tensor-core forward (one cooperative launch), 3 (backward only) the
 * backward for n other than 4 (tcgen05 dx and parameter-gradient kernels,
 * dx on the CUDA cores when D is not a multiple of 64; *cluster_size = the
 * token groups of its parameter-gradient kernel, *clusters = 2 when dx runs
 * in stream pairs (even n), 1 one 64-k block at a time, 0 on the CUDA
 * cores).  which = 0 forward: for
 * paths 1 and 2, *cluster_size is the number of K-slices the projection is
 * split into and *clusters the CTAs of its persistent grid.  which = 1 backward:
 * for path 1, the tensor-core kernel's grid is *clusters token groups of
 * *cluster_size d-slice CTAs each.  (No kernel uses thread-block clusters;
 * the parameter names are kept for ABI stability.)  No counterpart in the
 * reference (its Triton grids are fixed per call). */
MHC_API int mhc_query_plan(int which, int64_t tokens, int32_t n, int32_t D, int* path, int* cluster_size,
                           int* clusters);

/* The plan mhc_query_plan would report on an sm_100 device with `sms` SMs,
 * computed on the host without a device (capacity planning, host-side
 * tests).  It assumes the fused forward's cooperative launch fits, as it does
 * on every sm_100 part.  1 <= sms <= 4096.  No counterpart in the reference. */
MHC_API int mhc_query_plan_for(int which, int64_t tokens, int32_t n, int32_t D, int32_t sms, int* path,
                               int* cluster_size, int* clusters);

/* The grid of the n = 4 tensor-core backward (path 1 above) on a device with
 * `sms` SMs (sms = 0: the current device), written to grid[0..5]:
 * {Dc, S_K, S_T, J, E, R}.  S_K d-slices of Dc columns per stream times S_T
 * token groups of 128-token tiles; when the tiles do not split evenly and SMs
 * are left over, E > 0 more CTAs take the R leftover tiles (whole d-slices
 * each) and the S_K * S_T main CTAs J tiles each (E = J = R = 0: every tile
 * round robin over the token groups).  MHC_ERR_BAD_SHAPE for shapes that do
 * not take that path.  No counterpart in the reference (ABI 1.4.0). */
MHC_API int mhc_query_bwd_grid(int64_t tokens, int32_t n, int32_t D, int32_t sms, int32_t* grid);

/* mhc_bwd_workspace_size for a device with `sms` SMs, without a device. */
MHC_API int mhc_bwd_workspace_size_for(int64_t tokens, int32_t n, int32_t D, int32_t sms, size_t* bytes);

/* ---------------------------------------------------------------- post-op
 * The mHC post-op, the consumer of h_post and h_res: the next residual
 * stream of the hyper-connection block,
 *   out[t,i,:] = sum_j h_res[t,i,j] x[t,j,:] + h_post[t,i] y[t,:],
 * y = f(h_in) [T,D] bf16 the sublayer's output.  No counterpart in the
 * reference, which stops at h_post / h_res (src/forward/golden.py:65-69).
 * Shapes as above (1 <= n <= 8, D >= 1, T >= 0); no workspace.  The bf16
 * outputs are sums in ascending term order with each multiply and add
 * rounded on its own, then one round-to-nearest-even to bf16.  16-byte
 * aligned bf16 pointers with D a multiple of 8 take the vector kernels. */
typedef struct mhc_post_fwd_args {
  const uint16_t* x;       /* [T,n,D] bf16 */
  const float* h_res;      /* [T,n,n] */
  const float* h_post;     /* [T,n] */
  const uint16_t* y;       /* [T,D] bf16 */
  uint16_t* out;           /* [T,n,D] bf16 */
  int64_t tokens;
  int32_t n;
  int32_t D;
} mhc_post_fwd_args;

/* Backward of the post-op from dout [T,n,D] bf16:
 *   dx[t,j,:] = sum_i h_res[t,i,j] dout[t,i,:] (bf16), dy[t,:] = sum_i
 *   h_post[t,i] dout[t,i,:] (bf16), dh_res[t,i,j] = sum_d dout[t,i,d]
 *   x[t,j,d], dh_post[t,i] = sum_d dout[t,i,d] y[t,d] (fp32, summed in a
 *   fixed order, so repeated calls return identical bytes). */
typedef struct mhc_post_bwd_args {
  const uint16_t* x;
  const float* h_res;
  const float* h_post;
  const uint16_t* y;
  const uint16_t* dout;    /* [T,n,D] bf16 */
  uint16_t* dx;            /* [T,n,D] bf16 */
  uint16_t* dy;            /* [T,D] bf16 */
  float* dh_res;           /* [T,n,n] */
  float* dh_post;          /* [T,n] */
  int64_t tokens;
  int32_t n;
  int32_t D;
} mhc_post_bwd_args;

MHC_API int mhc_post_fwd(const mhc_post_fwd_args* args, void* stream);
MHC_API int mhc_post_bwd(const mhc_post_bwd_args* args, void* stream);

/* Number of kernels this library has launched in this process (all devices,
 * all threads).  No counterpart in the reference; used to report launches. */
MHC_API uint64_t mhc_launch_count(void);

/* Version of this ABI (major*10000 + minor*100 + patch).  1.1.0 added the
 * post-op and the device-free plan queries, 1.2.0 the backward that
 * recomputes the forward's intermediates and mhc_fwd_ex, 1.3.0 the
 * debug-bounds entry points, 1.4.0 mhc_query_bwd_grid. */
MHC_API int mhc_abi_version(void);

/* Debug-bounds builds (compiled with -DMHC_DEBUG_BOUNDS: lib/libmhc_ops_dbg.so
 * from `python -m mhc_ops_b200.build --debug-bounds`).  Every entry point
 * registers the buffers it was given (argument arrays with their byte sizes
 * and the workspace) before it launches, and every checked global access of
 * the kernels must lie inside one of them; one that does not is skipped --
 * nothing traps -- and the first is recorded.  mhc_debug_bounds synchronizes
 * the device, copies the record {count, site, address, bytes} of the calls
 * since the last clear into record[4] (site = file id * 100000 + source line
 * of the check) and clears it when clear != 0; it returns MHC_OK when count
 * is 0 and MHC_ERR_OUT_OF_BOUNDS otherwise.  One call at a time per process
 * (the buffer table is global), and not under stream capture.  Normal builds
 * check nothing and return MHC_ERR_UNSUPPORTED.  No counterpart in the
 * reference, which has no sanitizer path. */
MHC_API int mhc_debug_bounds(uint64_t* record, int clear);

/* Debug-bounds builds: runs one kernel that checks an address one byte past a
 * 256-byte buffer it registers inside `workspace` (no memory is accessed: the
 * check alone fails and is recorded), so a test can see the record path work.
 * Normal builds return MHC_ERR_UNSUPPORTED. */
MHC_API int mhc_debug_bounds_selftest(void* workspace, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MHC_OPS_H_ */
