"""Forward of the mHC pre-op on B200 -- drop-in for ``src/forward`` of the reference.

``mhc_forward_pre(x, phi, alpha, bias, outflag=False, norm_eps=1e-6, hc_eps=1e-6)``
keeps the reference signature and return convention (``src/forward/golden.py:10-69``):

* returns ``(h_in, h_post, h_res)``; with ``outflag`` also
  ``(inv_rms [B,S], h_mix [B,S,N], h_pre [B,S,n])``.
* ``h_in`` is bf16 ``[B,S,D]``; every other output is fp32.

It runs the sm_100a kernels of libmhc_ops.so through the C ABI on the current
CUDA stream.  CPU tensors raise (the reference's Triton wrapper silently fell
back to the golden, ``mhc_forward_pre_triton.py:423-425``; this build has no
fallback).  ``h_pre`` returned with ``outflag`` is the true gate value
(``golden.py:58``), not the reconstruction the reference's Triton wrappers used.
"""
from __future__ import annotations

import torch

from . import _lib

__all__ = ["mhc_forward_pre", "mhc_forward_pre_triton", "mhc_forward_pre_triton_optimized"]


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


def mhc_forward_pre(x, phi, alpha, bias, outflag: bool = False, norm_eps: float = 1e-6,
                    hc_eps: float = 1e-6):
    """mHC pre-op forward; see the module docstring."""
    _check_x(x)
    B, S, n, D = x.shape
    N = n * n + 2 * n
    dev = x.device
    x = x.contiguous()
    phi = _as_f32(phi, dev, "phi")
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

    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        lib = _lib.load()
        nbytes = _lib.fwd_workspace_size(T, n, D)
        ws = _lib.workspace(nbytes, dev, stream)
        args = _lib.FwdArgs(
            x=_lib.ptr(x), phi=_lib.ptr(phi), alpha=_lib.ptr(alpha), bias=_lib.ptr(bias),
            h_in=_lib.ptr(h_in), h_post=_lib.ptr(h_post), h_res=_lib.ptr(h_res),
            inv_rms=_lib.ptr(inv_rms), h_mix=_lib.ptr(h_mix), h_pre=_lib.ptr(h_pre),
            tokens=T, n=n, D=D, norm_eps=float(norm_eps), hc_eps=float(hc_eps),
            workspace=ws.buf.data_ptr(), workspace_bytes=ws.buf.numel())
        _lib.check(lib.mhc_fwd(args, stream.cuda_stream), "mhc_fwd")
        ws.watch(stream, "mhc_fwd")

    if not outflag:
        return h_in, h_post, h_res
    return h_in, h_post, h_res, inv_rms, h_mix, h_pre


# The reference exposes the same call under its Triton names
# (src/forward/__init__.py:7-11); they are the same B200 kernels here.
mhc_forward_pre_triton = mhc_forward_pre
mhc_forward_pre_triton_optimized = mhc_forward_pre
