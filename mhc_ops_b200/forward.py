"""Forward of the mHC pre-op on B200 -- drop-in for ``src/forward`` of the reference.

``mhc_forward_pre(x, phi, alpha, bias, outflag=False, norm_eps=1e-6, hc_eps=1e-6)``
keeps the reference signature and return convention (``src/forward/golden.py:10-69``):

* returns ``(h_in, h_post, h_res)``; with ``outflag`` also
  ``(inv_rms [B,S], h_mix [B,S,N], h_pre [B,S,n])``.
* ``h_in`` is bf16 ``[B,S,D]``; every other output is fp32.

It runs the sm_100a kernels of libmhc_ops.so through the C ABI on the current
CUDA stream.  CPU tensors raise (the reference's Triton wrapper silently fell
back to the golden, ``mhc_forward_pre_triton.py:423-425``; this library has no
fallback).  ``h_pre`` returned with ``outflag`` is the true gate value
(``golden.py:58``), not the reconstruction the reference's Triton wrappers used.
"""
from __future__ import annotations

import torch

from . import _lib

__all__ = ["mhc_forward_pre", "mhc_forward_pre_triton", "mhc_forward_pre_triton_optimized",
           "mhc_forward_pre_fused_norm", "mhc_forward_pre_fp8", "quantize_fp8_pow2"]


def _as_f32(t, device, name):
    if not torch.is_tensor(t):
        t = torch.as_tensor(t, dtype=torch.float32, device=device)
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, x is on {device}")
    return t.to(torch.float32).contiguous()


def _check_x(x: torch.Tensor) -> None:
    if not torch.is_tensor(x) or x.dim() != 4:
        raise ValueError("x must be a tensor of shape [B, S, n, D]")
    if not x.is_cuda:
        raise RuntimeError("mhc_ops_b200 runs on CUDA only: x is on the CPU (there is no CPU fallback)")
    if x.dtype != torch.bfloat16:
        raise TypeError(f"x must be bfloat16, got {x.dtype}")


def _forward(x, phi, alpha, bias, outflag, norm_eps, hc_eps, h_in_norm_eps, sm_budget=None, x_exp=None):
    fp8 = torch.is_tensor(x) and x.dtype == torch.float8_e4m3fn
    if fp8:
        if x.dim() != 4 or not x.is_cuda:
            raise ValueError("x_fp8 must be a CUDA tensor of shape [B, S, n, D]")
    else:
        _check_x(x)
    B, S, n, D = x.shape
    N = n * n + 2 * n
    dev = x.device
    x = x.contiguous()
    if x_exp is not None:
        if not fp8:
            raise ValueError("x_exp goes with an fp8 x")
        if tuple(x_exp.shape) != (B, S) or x_exp.dtype != torch.int8 or x_exp.device != dev:
            raise ValueError(f"x_exp must be an int8 [{B}, {S}] tensor on {dev}")
        x_exp = x_exp.contiguous()
    if not torch.is_tensor(phi) or phi.device != dev:
        raise ValueError(f"phi must be a tensor on {dev}")
    bf16_phi = phi.dtype == torch.bfloat16
    phi = phi.contiguous() if bf16_phi else _as_f32(phi, dev, "phi")
    alpha = _as_f32(alpha, dev, "alpha")
    bias = _as_f32(bias, dev, "bias")
    if tuple(phi.shape) != (N, n * D):
        raise ValueError(f"phi must be [{N}, {n * D}], got {tuple(phi.shape)}")
    if alpha.numel() != 3 or bias.numel() != N:
        raise ValueError("alpha must have 3 elements and bias n*n+2n")

    T = B * S
    h_in = torch.empty((B, S, D), dtype=torch.bfloat16, device=dev)
    h_post = torch.empty((B, S, n), dtype=torch.float32, device=dev)
    h_res = torch.empty((B, S, n, n), dtype=torch.float32, device=dev)
    inv_rms = h_mix = h_pre = None
    if outflag:
        inv_rms = torch.empty((B, S), dtype=torch.float32, device=dev)
        h_mix = torch.empty((B, S, N), dtype=torch.float32, device=dev)
        h_pre = torch.empty((B, S, n), dtype=torch.float32, device=dev)
    h_in_rstd = None if h_in_norm_eps is None else torch.empty((B, S), dtype=torch.float32, device=dev)
    ex = None
    if bf16_phi or h_in_rstd is not None or sm_budget or fp8:
        ex = _lib.FwdExArgs(phi_bf16=_lib.ptr(phi) if bf16_phi else None, h_in_rstd=_lib.ptr(h_in_rstd),
                            h_in_eps=float(h_in_norm_eps or 0.0), sm_budget=int(sm_budget or 0),
                            x_fp8=_lib.ptr(x) if fp8 else None, x_exp=_lib.ptr(x_exp))

    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        lib = _lib.load()
        nbytes = _lib.fwd_workspace_size(T, n, D, ex)
        ws = _lib.workspace(nbytes, dev, stream)
        args = _lib.FwdArgs(
            x=None if fp8 else _lib.ptr(x), phi=None if bf16_phi else _lib.ptr(phi), alpha=_lib.ptr(alpha),
            bias=_lib.ptr(bias),
            h_in=_lib.ptr(h_in), h_post=_lib.ptr(h_post), h_res=_lib.ptr(h_res),
            inv_rms=_lib.ptr(inv_rms), h_mix=_lib.ptr(h_mix), h_pre=_lib.ptr(h_pre),
            tokens=T, n=n, D=D, norm_eps=float(norm_eps), hc_eps=float(hc_eps),
            workspace=ws.buf.data_ptr(), workspace_bytes=ws.buf.numel())
        if ex is None:
            _lib.check(lib.mhc_fwd(args, stream.cuda_stream), "mhc_fwd")
        else:
            _lib.check(lib.mhc_fwd_ex(args, ex, stream.cuda_stream), "mhc_fwd_ex")
        ws.watch(stream, "mhc_fwd")
    return h_in, h_in_rstd, h_post, h_res, inv_rms, h_mix, h_pre


def mhc_forward_pre(x, phi, alpha, bias, outflag: bool = False, norm_eps: float = 1e-6,
                    hc_eps: float = 1e-6, sm_budget: int | None = None):
    """mHC pre-op forward; see the module docstring.  ``phi`` may be fp32 (the
    reference's type) or bf16 (then exact in one bf16 term: one tensor-core
    product per K-step instead of three).  ``sm_budget`` (not in the
    reference): the most SMs the forward's grids take, so that a collective
    left running on the other SMs overlaps it."""
    h_in, _, h_post, h_res, inv_rms, h_mix, h_pre = _forward(x, phi, alpha, bias, outflag, norm_eps, hc_eps, None,
                                                             sm_budget)
    if not outflag:
        return h_in, h_post, h_res
    return h_in, h_post, h_res, inv_rms, h_mix, h_pre


def mhc_forward_pre_fused_norm(x, phi, alpha, bias, h_in_norm_eps: float = 1e-6, outflag: bool = False,
                               norm_eps: float = 1e-6, hc_eps: float = 1e-6):
    """The forward fused with the statistic of the RMSNorm that opens the next
    sublayer: returns ``(h_in, h_in_rstd, h_post, h_res)`` (plus the outflag
    outputs), ``h_in_rstd [B,S] = 1 / sqrt(mean_d(h_in^2) + h_in_norm_eps)``
    over the bf16 ``h_in`` row, computed while ``h_in`` is written.  The next
    sublayer's ``RMSNorm(h_in) = h_in * h_in_rstd * weight`` then needs no
    reduction pass over ``h_in``.  No counterpart in the reference, whose
    forward stops at ``h_in`` (``src/forward/golden.py:62-63``)."""
    h_in, rstd, h_post, h_res, inv_rms, h_mix, h_pre = _forward(x, phi, alpha, bias, outflag, norm_eps, hc_eps,
                                                                h_in_norm_eps)
    if not outflag:
        return h_in, rstd, h_post, h_res
    return h_in, rstd, h_post, h_res, inv_rms, h_mix, h_pre


def mhc_forward_pre_fp8(x_fp8, x_exp, phi, alpha, bias, outflag: bool = False, norm_eps: float = 1e-6,
                        hc_eps: float = 1e-6):
    """Inference forward on an fp8 x: ``x_fp8`` float8_e4m3fn ``[B,S,n,D]`` and
    ``x_exp`` int8 ``[B,S]`` (or None for 0), ``x = x_fp8 * 2**x_exp`` per
    token (``quantize_fp8_pow2`` makes them from a bf16 x).  Every such value
    is exact in bf16, and the outputs equal, bit for bit, those of
    ``mhc_forward_pre`` on that bf16 x, while the forward reads half the bytes
    of x.  Same returns as ``mhc_forward_pre``.  Shapes the tensor-core
    forward takes only (n in {4, 8}, D a multiple of 64).  Not in the
    reference, whose x is bf16 (``src/forward/golden.py:38``)."""
    h_in, _, h_post, h_res, inv_rms, h_mix, h_pre = _forward(x_fp8, phi, alpha, bias, outflag, norm_eps, hc_eps,
                                                             None, None, x_exp)
    if not outflag:
        return h_in, h_post, h_res
    return h_in, h_post, h_res, inv_rms, h_mix, h_pre


def quantize_fp8_pow2(x: torch.Tensor):
    """bf16 x ``[B,S,n,D]`` -> (e4m3 x ``[B,S,n,D]``, int8 exponents ``[B,S]``)
    with one power-of-two scale per token, chosen so the token's largest
    magnitude fits e4m3's largest finite value (448).  Lossy (3 mantissa
    bits); ``x_fp8 * 2**x_exp`` is what ``mhc_forward_pre_fp8`` computes on."""
    B, S = x.shape[:2]
    amax = x.float().abs().reshape(B, S, -1).amax(-1).clamp_min(2.0 ** -100)
    e = torch.ceil(torch.log2(amax / 448.0)).clamp(-120, 120)
    x8 = (x.float() * torch.exp2(-e)[:, :, None, None]).to(torch.float8_e4m3fn)
    return x8, e.to(torch.int8)


# The reference exposes the same call under its Triton names
# (src/forward/__init__.py:7-11); they are the same B200 kernels here.
mhc_forward_pre_triton = mhc_forward_pre
mhc_forward_pre_triton_optimized = mhc_forward_pre
