"""Backward of the mHC pre-op on B200 -- drop-in for ``src/backward`` of the reference.

``mhc_backward_manual(x, phi, alpha, bias, inv_rms, h_mix, h_pre, h_post,
dh_in, dh_post, dh_res, gamma, norm_eps=1e-6, hc_eps=1e-6)`` keeps the
reference signature (``src/backward/golden.py:10-13``) and returns
``(dx bf16 [B,S,n,D], dphi [N,nD], dalpha [3], dbias [N], dgamma [nD])`` --
``dgamma`` flat, exactly as the golden returns it (``golden.py:93``).

``gamma`` may be ``None`` (all ones).  ``inv_rms``, ``h_mix`` and ``h_pre``
may all be ``None`` (and then ``h_post`` too): the forward's intermediates are
recomputed from ``x`` (the forward kernels run first inside the call, so a
forward that skipped ``outflag`` pays one more read of x instead of storing
116 bytes per token at n = 4); ``bias`` is then required.  The recomputed
values equal the ones ``mhc_forward_pre(..., outflag=True)`` returns bit for
bit, and so do the gradients.  The optional ``grad_out`` is a flat
fp32 buffer of ``N*nD + nD + 3 + N`` elements; when given, dphi, dgamma,
dalpha and dbias are written into it (in that order) and returned as views,
which lets a data-parallel caller all-reduce one buffer without a copy.
"""
from __future__ import annotations

import torch

from . import _lib
from .forward import _as_f32, _check_x

__all__ = ["mhc_backward_manual", "mhc_backward_triton", "param_grad_numel", "split_param_grads"]


def param_grad_numel(n: int, D: int) -> int:
    N = n * n + 2 * n
    return N * n * D + n * D + 3 + N


def split_param_grads(flat: torch.Tensor, n: int, D: int):
    """Views (dphi [N,nD], dgamma [nD], dalpha [3], dbias [N]) into a flat grad buffer."""
    N = n * n + 2 * n
    nD = n * D
    o = 0
    dphi = flat[o:o + N * nD].view(N, nD); o += N * nD
    dgamma = flat[o:o + nD]; o += nD
    dalpha = flat[o:o + 3]; o += 3
    dbias = flat[o:o + N]
    return dphi, dgamma, dalpha, dbias


def mhc_backward_manual(x, phi, alpha, bias, inv_rms, h_mix, h_pre, h_post, dh_in, dh_post, dh_res,
                        gamma, norm_eps: float = 1e-6, hc_eps: float = 1e-6, grad_out=None):
    """mHC pre-op backward; see the module docstring."""
    _check_x(x)
    B, S, n, D = x.shape
    N = n * n + 2 * n
    nD = n * D
    T = B * S
    dev = x.device
    x = x.contiguous()
    phi = _as_f32(phi, dev, "phi")
    alpha = _as_f32(alpha, dev, "alpha")
    recompute = inv_rms is None and h_mix is None and h_pre is None
    if recompute:
        if bias is None:
            raise ValueError("recomputing the forward's intermediates needs bias")
        bias = _as_f32(bias, dev, "bias")
        if bias.numel() != N:
            raise ValueError("bias must have n*n+2n elements")
    elif inv_rms is None or h_mix is None or h_pre is None or h_post is None:
        raise ValueError("give inv_rms, h_mix, h_pre and h_post, or None for the first three to recompute them")
    else:
        inv_rms = _as_f32(inv_rms, dev, "inv_rms")
        h_mix = _as_f32(h_mix, dev, "h_mix")
        h_pre = _as_f32(h_pre, dev, "h_pre")
    h_post = None if h_post is None else _as_f32(h_post, dev, "h_post")
    dh_post = _as_f32(dh_post, dev, "dh_post")
    dh_res = _as_f32(dh_res, dev, "dh_res")
    gamma = None if gamma is None else _as_f32(gamma, dev, "gamma")
    if not torch.is_tensor(dh_in) or dh_in.device != dev:
        raise ValueError("dh_in must be a tensor on x's device")
    dh_in = dh_in.to(torch.bfloat16).contiguous()
    checks = [(phi, (N, nD)), (inv_rms, (B, S)), (h_mix, (B, S, N)), (h_pre, (B, S, n)),
              (h_post, (B, S, n)), (dh_in, (B, S, D)), (dh_post, (B, S, n)), (dh_res, (B, S, n, n))]
    for t, shp in checks:
        if t is not None and tuple(t.shape) != shp:
            raise ValueError(f"expected shape {shp}, got {tuple(t.shape)}")
    if gamma is not None and gamma.numel() != nD:
        raise ValueError(f"gamma must have n*D = {nD} elements")
    if alpha.numel() != 3:
        raise ValueError("alpha must have 3 elements")

    dx = torch.empty((B, S, n, D), dtype=torch.bfloat16, device=dev)
    if grad_out is None:
        grad_out = torch.empty(param_grad_numel(n, D), dtype=torch.float32, device=dev)
    elif (grad_out.dtype != torch.float32 or grad_out.device != dev or not grad_out.is_contiguous()
          or grad_out.numel() != param_grad_numel(n, D)):
        raise ValueError("grad_out must be a contiguous fp32 buffer of param_grad_numel(n, D) elements")
    dphi, dgamma, dalpha, dbias = split_param_grads(grad_out, n, D)

    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        lib = _lib.load()
        nbytes = _lib.bwd_workspace_size(T, n, D, recompute=recompute)
        ws = _lib.workspace(nbytes, dev, stream)
        args = _lib.BwdArgs(
            x=_lib.ptr(x), phi=_lib.ptr(phi), alpha=_lib.ptr(alpha), bias=_lib.ptr(bias) if recompute else None,
            inv_rms=_lib.ptr(inv_rms), h_mix=_lib.ptr(h_mix), h_pre=_lib.ptr(h_pre), h_post=_lib.ptr(h_post),
            dh_in=_lib.ptr(dh_in), dh_post=_lib.ptr(dh_post), dh_res=_lib.ptr(dh_res), gamma=_lib.ptr(gamma),
            dx=_lib.ptr(dx), dphi=_lib.ptr(dphi), dalpha=_lib.ptr(dalpha), dbias=_lib.ptr(dbias),
            dgamma=_lib.ptr(dgamma), tokens=T, n=n, D=D, norm_eps=float(norm_eps), hc_eps=float(hc_eps),
            workspace=ws.buf.data_ptr(), workspace_bytes=ws.buf.numel())
        _lib.check(lib.mhc_bwd(args, stream.cuda_stream), "mhc_bwd")
        ws.watch(stream, "mhc_bwd")
    return dx, dphi, dalpha, dbias, dgamma


# The reference's Triton name for the same call (src/backward/__init__.py:7-8).
mhc_backward_triton = mhc_backward_manual
