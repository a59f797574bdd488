"""CPU oracle for the mHC post-op (forward and backward).  TEST INFRASTRUCTURE ONLY.

Imported only by ``tests/`` and ``bench.py``'s measurement of the post-op, as
the checker; the product path (``mhc_ops_b200.post``) never imports it.

Parity unpinned: the reference (folrent1896/mhc_ops) has no post-op -- it
stops at ``h_post`` / ``h_res`` (``src/forward/golden.py:65-69``) -- so there
is no golden to pin against.  This module restates the hyper-connection
update ``x_next = h_res x + h_post y`` (the step after the pre-op in an mHC
block) and its gradient; ``tests/test_post_oracle.py`` checks it against
torch autograd in float64 on the CPU, an independent derivation.

Operation order (what the CUDA kernels follow, so the bf16 results match
bit for bit): float32, every multiply and every add rounded on its own, terms
in ascending index order, then one round-to-nearest-even to bf16.  The fp32
row sums (dh_res, dh_post) are float64 sums of exact bf16 x bf16 products,
rounded once to float32; the kernels sum in another fixed order, so those are
compared with a tolerance.
"""
from __future__ import annotations

import numpy as np

from .mhc_oracle import bf16_to_f32, f32_to_bf16

__all__ = ["post_forward", "post_backward"]


def post_forward(x_bf16, h_res, h_post, y_bf16):
    """x [T,n,D] u16, h_res [T,n,n] f32, h_post [T,n] f32, y [T,D] u16 -> out [T,n,D] u16."""
    x = bf16_to_f32(x_bf16)
    y = bf16_to_f32(y_bf16)
    h_res = np.asarray(h_res, np.float32)
    h_post = np.asarray(h_post, np.float32)
    n = x.shape[1]
    out = np.empty_like(x)
    for i in range(n):
        acc = h_res[:, i, 0:1] * x[:, 0, :]
        for j in range(1, n):
            acc = acc + h_res[:, i, j:j + 1] * x[:, j, :]
        out[:, i, :] = acc + h_post[:, i:i + 1] * y
    return f32_to_bf16(out)


def post_backward(x_bf16, h_res, h_post, y_bf16, dout_bf16):
    """-> (dx [T,n,D] u16, dh_res [T,n,n] f32, dh_post [T,n] f32, dy [T,D] u16)."""
    x = bf16_to_f32(x_bf16)
    y = bf16_to_f32(y_bf16)
    g = bf16_to_f32(dout_bf16)
    h_res = np.asarray(h_res, np.float32)
    h_post = np.asarray(h_post, np.float32)
    n = x.shape[1]
    dx = np.empty_like(x)
    for j in range(n):
        acc = h_res[:, 0, j:j + 1] * g[:, 0, :]
        for i in range(1, n):
            acc = acc + h_res[:, i, j:j + 1] * g[:, i, :]
        dx[:, j, :] = acc
    dy = h_post[:, 0:1] * g[:, 0, :]
    for i in range(1, n):
        dy = dy + h_post[:, i:i + 1] * g[:, i, :]
    g64, x64, y64 = g.astype(np.float64), x.astype(np.float64), y.astype(np.float64)
    dh_res = np.einsum("tid,tjd->tij", g64, x64).astype(np.float32)
    dh_post = np.einsum("tid,td->ti", g64, y64).astype(np.float32)
    return f32_to_bf16(dx), dh_res, dh_post, f32_to_bf16(dy)


def post_backward_term_scale(x_bf16, y_bf16, dout_bf16):
    """sum |terms| of dh_res and dh_post (the scale of their summation error)."""
    x = np.abs(bf16_to_f32(x_bf16).astype(np.float64))
    y = np.abs(bf16_to_f32(y_bf16).astype(np.float64))
    g = np.abs(bf16_to_f32(dout_bf16).astype(np.float64))
    return np.einsum("tid,tjd->tij", g, x), np.einsum("tid,td->ti", g, y)
