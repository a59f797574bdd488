"""The mHC post-op on B200: the consumer of the pre-op's ``h_post`` / ``h_res``.

A hyper-connection block turns its n residual streams ``x [B,S,n,D]`` into
``h_in`` (the pre-op), runs the sublayer ``y = f(h_in) [B,S,D]`` and writes
the next streams

    x_next[..., i, :] = sum_j h_res[..., i, j] x[..., j, :] + h_post[..., i] y

The reference stops at ``h_post`` / ``h_res`` (``src/forward/golden.py:65-69``);
this module adds that next step, forward and backward, on the sm_100a kernels
of libmhc_ops.so (``mhc_post_fwd`` / ``mhc_post_bwd`` of the C ABI), and an
autograd Function over both.  bf16 in and out for the streams and y, fp32
for the coefficients and their gradients; CPU tensors raise.
"""
from __future__ import annotations

import torch

from . import _lib

__all__ = ["mhc_post", "mhc_post_backward", "MHCPostFunction", "mhc_post_fn"]


def _check(x, h_res, h_post, y):
    if not torch.is_tensor(x) or x.dim() != 4:
        raise ValueError("x must be a tensor of shape [B, S, n, D]")
    if not x.is_cuda:
        raise RuntimeError("mhc_ops_b200 runs on CUDA only: x is on the CPU (there is no CPU fallback)")
    B, S, n, D = x.shape
    if x.dtype != torch.bfloat16 or y.dtype != torch.bfloat16:
        raise TypeError("x and y must be bfloat16")
    if tuple(y.shape) != (B, S, D):
        raise ValueError(f"y must be [{B}, {S}, {D}], got {tuple(y.shape)}")
    if tuple(h_res.shape) != (B, S, n, n) or tuple(h_post.shape) != (B, S, n):
        raise ValueError("h_res must be [B, S, n, n] and h_post [B, S, n]")
    for t, name in ((y, "y"), (h_res, "h_res"), (h_post, "h_post")):
        if t.device != x.device:
            raise ValueError(f"{name} is on {t.device}, x is on {x.device}")
    return B, S, n, D


def mhc_post(x, h_res, h_post, y):
    """x_next = h_res @ x + h_post (outer) y, bf16 ``[B,S,n,D]``."""
    B, S, n, D = _check(x, h_res, h_post, y)
    dev = x.device
    x, y = x.contiguous(), y.contiguous()
    h_res = h_res.to(torch.float32).contiguous()
    h_post = h_post.to(torch.float32).contiguous()
    out = torch.empty_like(x)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        args = _lib.PostFwdArgs(x=_lib.ptr(x), h_res=_lib.ptr(h_res), h_post=_lib.ptr(h_post), y=_lib.ptr(y),
                                out=_lib.ptr(out), tokens=B * S, n=n, D=D)
        _lib.check(_lib.load().mhc_post_fwd(args, stream.cuda_stream), "mhc_post_fwd")
    return out


def mhc_post_backward(x, h_res, h_post, y, dout):
    """Gradients ``(dx, dh_res, dh_post, dy)`` of ``mhc_post`` for the upstream ``dout``."""
    B, S, n, D = _check(x, h_res, h_post, y)
    if tuple(dout.shape) != (B, S, n, D):
        raise ValueError(f"dout must be [{B}, {S}, {n}, {D}], got {tuple(dout.shape)}")
    dev = x.device
    x, y = x.contiguous(), y.contiguous()
    dout = dout.to(torch.bfloat16).contiguous()
    h_res = h_res.to(torch.float32).contiguous()
    h_post = h_post.to(torch.float32).contiguous()
    dx = torch.empty_like(x)
    dy = torch.empty_like(y)
    dh_res = torch.empty((B, S, n, n), dtype=torch.float32, device=dev)
    dh_post = torch.empty((B, S, n), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev)
        args = _lib.PostBwdArgs(x=_lib.ptr(x), h_res=_lib.ptr(h_res), h_post=_lib.ptr(h_post), y=_lib.ptr(y),
                                dout=_lib.ptr(dout), dx=_lib.ptr(dx), dy=_lib.ptr(dy), dh_res=_lib.ptr(dh_res),
                                dh_post=_lib.ptr(dh_post), tokens=B * S, n=n, D=D)
        _lib.check(_lib.load().mhc_post_bwd(args, stream.cuda_stream), "mhc_post_bwd")
    return dx, dh_res, dh_post, dy


class MHCPostFunction(torch.autograd.Function):
    """autograd over ``mhc_post``: gradients for x, h_res, h_post and y."""

    @staticmethod
    def forward(ctx, x, h_res, h_post, y):
        ctx.save_for_backward(x, h_res, h_post, y)
        return mhc_post(x, h_res, h_post, y)

    @staticmethod
    def backward(ctx, dout):
        x, h_res, h_post, y = ctx.saved_tensors
        dx, dh_res, dh_post, dy = mhc_post_backward(x, h_res, h_post, y, dout)
        return dx, dh_res.to(h_res.dtype), dh_post.to(h_post.dtype), dy


def mhc_post_fn(x, h_res, h_post, y):
    return MHCPostFunction.apply(x, h_res, h_post, y)
