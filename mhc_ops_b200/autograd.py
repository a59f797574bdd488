"""``torch.autograd.Function`` wrapper of the mHC pre-op (absent from the reference).

The reference leaves training to the user: call the forward with
``outflag=True`` and pass the intermediates into ``mhc_backward_manual`` by
hand (reference ``README.md:200-224``).  ``MHCPreFunction`` does that wiring.

gamma semantics.  The reference backward takes a ``gamma [n, D]``
(``src/backward/golden.py:68,94``) that its forward does not.  The golden
backward is exactly the gradient of the forward evaluated with
``phi_eff = phi * gamma.reshape(1, nD)`` -- gamma scales x inside the
projection only; the RMS uses plain x.  So the autograd forward folds gamma
into phi and the backward returns gradients for x, phi, alpha, bias and gamma.
With ``gamma=None`` the fold is skipped and no gamma gradient is produced.

Both directions run as the registered operators ``torch.ops.mhc.fwd`` /
``torch.ops.mhc.bwd`` (``mhc_ops_b200.ops``), so ``torch.compile`` traces
``mhc_pre`` with each direction as one graph node.
"""
from __future__ import annotations

import torch

from . import ops

__all__ = ["MHCPreFunction", "mhc_pre"]


class MHCPreFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, phi, alpha, bias, gamma=None, norm_eps=1e-6, hc_eps=1e-6):
        n, D = x.shape[2], x.shape[3]
        phi_eff = phi if gamma is None else phi * gamma.reshape(1, n * D).to(phi.dtype)
        h_in, h_post, h_res, inv_rms, h_mix, h_pre = ops.fwd(x, phi_eff, alpha, bias, norm_eps, hc_eps)
        ctx.save_for_backward(x, phi, alpha, bias, gamma, inv_rms, h_mix, h_pre, h_post)
        ctx.eps = (norm_eps, hc_eps)
        ctx.shapes = (phi.dtype, alpha.dtype, bias.dtype)
        return h_in, h_post, h_res

    @staticmethod
    def backward(ctx, dh_in, dh_post, dh_res):
        x, phi, alpha, bias, gamma, inv_rms, h_mix, h_pre, h_post = ctx.saved_tensors
        norm_eps, hc_eps = ctx.eps
        if dh_in is None:
            dh_in = torch.zeros(x.shape[0], x.shape[1], x.shape[3], dtype=torch.bfloat16, device=x.device)
        if dh_post is None:
            dh_post = torch.zeros_like(h_post)
        if dh_res is None:
            n = x.shape[2]
            dh_res = torch.zeros(x.shape[0], x.shape[1], n, n, dtype=torch.float32, device=x.device)
        dx, dphi, dalpha, dbias, dgamma = ops.bwd(
            x, phi, alpha, inv_rms, h_mix, h_pre, h_post, dh_in.to(torch.bfloat16), dh_post, dh_res, gamma,
            norm_eps, hc_eps)
        g_gamma = None if gamma is None else dgamma.reshape(gamma.shape).to(gamma.dtype)
        return (dx, dphi.to(phi.dtype), dalpha.to(alpha.dtype), dbias.to(bias.dtype), g_gamma, None, None)


def mhc_pre(x, phi, alpha, bias, gamma=None, norm_eps: float = 1e-6, hc_eps: float = 1e-6):
    """Differentiable mHC pre-op: returns (h_in, h_post, h_res)."""
    return MHCPreFunction.apply(x, phi, alpha, bias, gamma, norm_eps, hc_eps)
