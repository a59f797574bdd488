// TORCH_LIBRARY(mhc, ...): the mHC pre-op as registered torch operators over
// the C ABI of libmhc_ops.so (include/mhc_ops.h).
//
//   mhc::fwd(x, phi, alpha, bias, norm_eps, hc_eps)
//       -> (h_in, h_post, h_res, inv_rms, h_mix, h_pre)
//     the reference's mhc_forward_pre(..., outflag=True)
//     (src/forward/golden.py:10-69; Triton call site
//     src/forward/mhc_forward_pre_triton.py:409-417);
//   mhc::bwd(x, phi, alpha, inv_rms, h_mix, h_pre, h_post, dh_in, dh_post,
//            dh_res, gamma?, norm_eps, hc_eps) -> (dx, dphi, dalpha, dbias, dgamma)
//     the reference's mhc_backward_manual (src/backward/golden.py:10-96;
//     Triton call site src/backward/mhc_backward_triton.py:467-473).
//
// CUDA kernels convert tensors to the ABI's argument structs, allocate the
// outputs, launch on at::cuda::getCurrentCUDAStream() and turn error codes
// into TORCH_CHECK failures.  There is no CPU kernel: CPU tensors fail in the
// dispatcher.  Meta kernels give the output shapes, so FakeTensor tracing
// (torch.compile, torch.export) sees the ops without running them.
//
// Workspaces are cached per (device, stream) and zero-filled once.  After
// every call the workspace's device status word (set when a kernel's bounded
// wait expired) is copied to pinned host memory on a side stream, without
// making the caller's stream wait; the next call through the same workspace,
// or mhc::check_status, reports it as an error.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/library.h>

#include <map>
#include <memory>
#include <mutex>
#include <tuple>
#include <utility>

#include "mhc_ops.h"

namespace {

void check_cuda(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

void check_status(int st, const char* where) {
  TORCH_CHECK(st == MHC_OK, where, ": mhc status ", st, ": ", mhc_status_string(st),
              st == MHC_ERR_CUDA ? std::string(" (") + mhc_last_cuda_error() + ")" : std::string());
}

// One cached workspace and the watch over its status word.
struct Workspace {
  at::Tensor buf;
  int* host = nullptr;          // pinned copy of the status word
  cudaStream_t side = nullptr;  // where the copy runs
  cudaEvent_t call_done = nullptr, copied = nullptr;
  bool pending = false;
  const char* where = "";

  ~Workspace() {
    // Process teardown may already have unloaded CUDA; errors are ignored.
    if (copied) cudaEventDestroy(copied);
    if (call_done) cudaEventDestroy(call_done);
    if (side) cudaStreamDestroy(side);
    if (host) cudaFreeHost(host);
  }

  void init(int64_t nbytes, const at::Device& dev) {
    buf = at::zeros({std::max<int64_t>(nbytes, 1 << 16)}, at::TensorOptions().dtype(at::kByte).device(dev));
    if (!host) {
      check_cuda(cudaHostAlloc(reinterpret_cast<void**>(&host), sizeof(int), cudaHostAllocDefault), "cudaHostAlloc");
      *host = 0;
      check_cuda(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking), "cudaStreamCreate");
      check_cuda(cudaEventCreateWithFlags(&call_done, cudaEventDisableTiming), "cudaEventCreate");
      check_cuda(cudaEventCreateWithFlags(&copied, cudaEventDisableTiming), "cudaEventCreate");
    }
  }

  // Raise if an earlier call reported an expired device wait (its outputs are
  // invalid); the word is cleared first.  wait: block until the last copy lands.
  void raise_if_timed_out(cudaStream_t stream, bool wait) {
    if (!pending) return;
    if (wait) {
      check_cuda(cudaEventSynchronize(copied), "cudaEventSynchronize");
    } else if (cudaEventQuery(copied) != cudaSuccess) {
      (void)cudaGetLastError();   // cudaErrorNotReady: look again at the next call
      return;
    }
    pending = false;
    const int code = *host;
    if (code != MHC_OK) {
      *host = 0;
      check_cuda(cudaMemsetAsync(buf.data_ptr(), 0, sizeof(int), stream), "cudaMemsetAsync");
      check_status(code, (std::string(where) + " (an earlier call; its outputs are invalid)").c_str());
    }
  }

  void watch(cudaStream_t stream, const char* name) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    check_cuda(cudaStreamIsCapturing(stream, &cap), "cudaStreamIsCapturing");
    if (cap != cudaStreamCaptureStatusNone) return;   // no host-visible copy inside a graph capture
    where = name;
    check_cuda(cudaEventRecord(call_done, stream), "cudaEventRecord");
    check_cuda(cudaStreamWaitEvent(side, call_done, 0), "cudaStreamWaitEvent");
    check_cuda(cudaMemcpyAsync(host, buf.data_ptr(), sizeof(int), cudaMemcpyDeviceToHost, side), "cudaMemcpyAsync");
    check_cuda(cudaEventRecord(copied, side), "cudaEventRecord");
    pending = true;
  }
};

std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, std::unique_ptr<Workspace>> g_ws;

Workspace& workspace(int64_t nbytes, const at::Device& dev, cudaStream_t stream) {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  auto& slot = g_ws[{dev.index(), stream}];
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  check_cuda(cudaStreamIsCapturing(stream, &cap), "cudaStreamIsCapturing");
  if (cap != cudaStreamCaptureStatusNone) {
    // inside a CUDA graph capture nothing may be allocated or synchronised:
    // the workspace must come from a call on this stream before the capture
    TORCH_CHECK(slot && slot->buf.defined() && slot->buf.numel() >= nbytes,
                "mhc: no workspace for this stream while it is capturing a CUDA graph; run the same call once "
                "on the capturing stream before the capture");
    return *slot;
  }
  if (!slot) slot = std::make_unique<Workspace>();
  if (slot->buf.defined()) slot->raise_if_timed_out(stream, /*wait=*/slot->buf.numel() < nbytes);
  if (!slot->buf.defined() || slot->buf.numel() < nbytes) slot->init(nbytes, dev);
  return *slot;
}

at::Tensor f32(const at::Tensor& t, const at::Device& dev, const char* name) {
  TORCH_CHECK(t.device() == dev, name, " is on ", t.device(), ", x is on ", dev);
  return t.to(at::kFloat).contiguous();
}

void check_x(const at::Tensor& x) {
  TORCH_CHECK(x.dim() == 4, "x must be [B, S, n, D]");
  TORCH_CHECK(x.is_cuda(), "mhc ops run on CUDA only (there is no CPU fallback)");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "x must be bfloat16, got ", x.scalar_type());
}

void check_shape(const at::Tensor& t, at::IntArrayRef want, const char* name) {
  TORCH_CHECK(t.sizes() == want, name, " must be ", want, ", got ", t.sizes());
}

}  // namespace

// ----------------------------------------------------------------- CUDA kernels
std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> mhc_fwd_cuda(
    const at::Tensor& x_in, const at::Tensor& phi_in, const at::Tensor& alpha_in, const at::Tensor& bias_in,
    double norm_eps, double hc_eps) {
  check_x(x_in);
  const at::Device dev = x_in.device();
  c10::cuda::CUDAGuard guard(dev);
  const int64_t B = x_in.size(0), S = x_in.size(1), n = x_in.size(2), D = x_in.size(3);
  const int64_t N = n * n + 2 * n, T = B * S;
  const at::Tensor x = x_in.contiguous();
  const at::Tensor phi = f32(phi_in, dev, "phi"), alpha = f32(alpha_in, dev, "alpha"), bias = f32(bias_in, dev, "bias");
  check_shape(phi, {N, n * D}, "phi");
  TORCH_CHECK(alpha.numel() == 3 && bias.numel() == N, "alpha must have 3 elements and bias n*n+2n");
  const auto o = x.options();
  at::Tensor h_in = at::empty({B, S, D}, o);
  at::Tensor h_post = at::empty({B, S, n}, o.dtype(at::kFloat));
  at::Tensor h_res = at::empty({B, S, n, n}, o.dtype(at::kFloat));
  at::Tensor inv_rms = at::empty({B, S}, o.dtype(at::kFloat));
  at::Tensor h_mix = at::empty({B, S, N}, o.dtype(at::kFloat));
  at::Tensor h_pre = at::empty({B, S, n}, o.dtype(at::kFloat));
  size_t nbytes = 0;
  check_status(mhc_fwd_workspace_size(T, (int32_t)n, (int32_t)D, &nbytes), "mhc_fwd_workspace_size");
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev.index()).stream();
  Workspace& ws = workspace((int64_t)nbytes, dev, stream);
  mhc_fwd_args a{};
  a.x = static_cast<const uint16_t*>(x.data_ptr());
  a.phi = phi.data_ptr<float>();
  a.alpha = alpha.data_ptr<float>();
  a.bias = bias.data_ptr<float>();
  a.h_in = static_cast<uint16_t*>(h_in.data_ptr());
  a.h_post = h_post.data_ptr<float>();
  a.h_res = h_res.data_ptr<float>();
  a.inv_rms = inv_rms.data_ptr<float>();
  a.h_mix = h_mix.data_ptr<float>();
  a.h_pre = h_pre.data_ptr<float>();
  a.tokens = T;
  a.n = (int32_t)n;
  a.D = (int32_t)D;
  a.norm_eps = (float)norm_eps;
  a.hc_eps = (float)hc_eps;
  a.workspace = ws.buf.data_ptr();
  a.workspace_bytes = (size_t)ws.buf.numel();
  check_status(mhc_fwd(&a, stream), "mhc::fwd");
  ws.watch(stream, "mhc::fwd");
  return {h_in, h_post, h_res, inv_rms, h_mix, h_pre};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> mhc_bwd_cuda(
    const at::Tensor& x_in, const at::Tensor& phi_in, const at::Tensor& alpha_in, const at::Tensor& inv_rms_in,
    const at::Tensor& h_mix_in, const at::Tensor& h_pre_in, const at::Tensor& h_post_in, const at::Tensor& dh_in_in,
    const at::Tensor& dh_post_in, const at::Tensor& dh_res_in, const c10::optional<at::Tensor>& gamma_in,
    double norm_eps, double hc_eps) {
  check_x(x_in);
  const at::Device dev = x_in.device();
  c10::cuda::CUDAGuard guard(dev);
  const int64_t B = x_in.size(0), S = x_in.size(1), n = x_in.size(2), D = x_in.size(3);
  const int64_t N = n * n + 2 * n, nD = n * D, T = B * S;
  const at::Tensor x = x_in.contiguous();
  const at::Tensor phi = f32(phi_in, dev, "phi"), alpha = f32(alpha_in, dev, "alpha");
  const at::Tensor inv_rms = f32(inv_rms_in, dev, "inv_rms"), h_mix = f32(h_mix_in, dev, "h_mix");
  const at::Tensor h_pre = f32(h_pre_in, dev, "h_pre"), h_post = f32(h_post_in, dev, "h_post");
  const at::Tensor dh_post = f32(dh_post_in, dev, "dh_post"), dh_res = f32(dh_res_in, dev, "dh_res");
  TORCH_CHECK(dh_in_in.device() == dev, "dh_in must be on x's device");
  const at::Tensor dh_in = dh_in_in.to(at::kBFloat16).contiguous();
  at::Tensor gamma;
  if (gamma_in.has_value() && gamma_in->defined()) {
    gamma = f32(*gamma_in, dev, "gamma");
    TORCH_CHECK(gamma.numel() == nD, "gamma must have n*D elements");
  }
  check_shape(phi, {N, nD}, "phi");
  check_shape(inv_rms, {B, S}, "inv_rms");
  check_shape(h_mix, {B, S, N}, "h_mix");
  check_shape(h_pre, {B, S, n}, "h_pre");
  check_shape(h_post, {B, S, n}, "h_post");
  check_shape(dh_in, {B, S, D}, "dh_in");
  check_shape(dh_post, {B, S, n}, "dh_post");
  check_shape(dh_res, {B, S, n, n}, "dh_res");
  TORCH_CHECK(alpha.numel() == 3, "alpha must have 3 elements");
  const auto o = x.options();
  at::Tensor dx = at::empty({B, S, n, D}, o);
  at::Tensor dphi = at::empty({N, nD}, o.dtype(at::kFloat));
  at::Tensor dalpha = at::empty({3}, o.dtype(at::kFloat));
  at::Tensor dbias = at::empty({N}, o.dtype(at::kFloat));
  at::Tensor dgamma = at::empty({nD}, o.dtype(at::kFloat));
  size_t nbytes = 0;
  check_status(mhc_bwd_workspace_size(T, (int32_t)n, (int32_t)D, &nbytes), "mhc_bwd_workspace_size");
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev.index()).stream();
  Workspace& ws = workspace((int64_t)nbytes, dev, stream);
  mhc_bwd_args a{};
  a.x = static_cast<const uint16_t*>(x.data_ptr());
  a.phi = phi.data_ptr<float>();
  a.alpha = alpha.data_ptr<float>();
  a.bias = nullptr;
  a.inv_rms = inv_rms.data_ptr<float>();
  a.h_mix = h_mix.data_ptr<float>();
  a.h_pre = h_pre.data_ptr<float>();
  a.h_post = h_post.data_ptr<float>();
  a.dh_in = static_cast<const uint16_t*>(dh_in.data_ptr());
  a.dh_post = dh_post.data_ptr<float>();
  a.dh_res = dh_res.data_ptr<float>();
  a.gamma = gamma.defined() ? gamma.data_ptr<float>() : nullptr;
  a.dx = static_cast<uint16_t*>(dx.data_ptr());
  a.dphi = dphi.data_ptr<float>();
  a.dalpha = dalpha.data_ptr<float>();
  a.dbias = dbias.data_ptr<float>();
  a.dgamma = dgamma.data_ptr<float>();
  a.tokens = T;
  a.n = (int32_t)n;
  a.D = (int32_t)D;
  a.norm_eps = (float)norm_eps;
  a.hc_eps = (float)hc_eps;
  a.workspace = ws.buf.data_ptr();
  a.workspace_bytes = (size_t)ws.buf.numel();
  check_status(mhc_bwd(&a, stream), "mhc::bwd");
  ws.watch(stream, "mhc::bwd");
  return {dx, dphi, dalpha, dbias, dgamma};
}

// Waits for the status copies of every workspace of the op layer and raises
// if any call reported an expired device wait.
int64_t mhc_check_status() {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  for (auto& kv : g_ws) {
    c10::cuda::CUDAGuard guard(kv.first.first);
    if (kv.second->buf.defined()) kv.second->raise_if_timed_out(kv.first.second, /*wait=*/true);
  }
  return 0;
}

// ----------------------------------------------------------------- Meta kernels (shapes only)
std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> mhc_fwd_meta(
    const at::Tensor& x, const at::Tensor& phi, const at::Tensor& alpha, const at::Tensor& bias, double, double) {
  TORCH_CHECK(x.dim() == 4, "x must be [B, S, n, D]");
  const auto B = x.sym_size(0), S = x.sym_size(1), n = x.sym_size(2), D = x.sym_size(3);
  const auto N = n * n + 2 * n;
  const auto f = x.options().dtype(at::kFloat);
  return {at::empty_symint({B, S, D}, x.options()), at::empty_symint({B, S, n}, f),
          at::empty_symint({B, S, n, n}, f), at::empty_symint({B, S}, f), at::empty_symint({B, S, N}, f),
          at::empty_symint({B, S, n}, f)};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> mhc_bwd_meta(
    const at::Tensor& x, const at::Tensor& phi, const at::Tensor&, const at::Tensor&, const at::Tensor&,
    const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
    const c10::optional<at::Tensor>&, double, double) {
  TORCH_CHECK(x.dim() == 4, "x must be [B, S, n, D]");
  const auto n = x.sym_size(2), D = x.sym_size(3);
  const auto N = n * n + 2 * n;
  const auto f = x.options().dtype(at::kFloat);
  return {at::empty_symint(x.sym_sizes(), x.options()), at::empty_symint({N, n * D}, f), at::empty_symint({3}, f),
          at::empty_symint({N}, f), at::empty_symint({n * D}, f)};
}

TORCH_LIBRARY(mhc, m) {
  m.def("fwd(Tensor x, Tensor phi, Tensor alpha, Tensor bias, float norm_eps=1e-6, float hc_eps=1e-6) -> "
        "(Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def("bwd(Tensor x, Tensor phi, Tensor alpha, Tensor inv_rms, Tensor h_mix, Tensor h_pre, Tensor h_post, "
        "Tensor dh_in, Tensor dh_post, Tensor dh_res, Tensor? gamma, float norm_eps=1e-6, float hc_eps=1e-6) -> "
        "(Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def("check_status() -> int");
  m.impl("check_status", &mhc_check_status);
}

TORCH_LIBRARY_IMPL(mhc, CUDA, m) {
  m.impl("fwd", &mhc_fwd_cuda);
  m.impl("bwd", &mhc_bwd_cuda);
}

TORCH_LIBRARY_IMPL(mhc, Meta, m) {
  m.impl("fwd", &mhc_fwd_meta);
  m.impl("bwd", &mhc_bwd_meta);
}
