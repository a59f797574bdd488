"""The post-op kernels (mhc_post_fwd / mhc_post_bwd of the C ABI) against the
post-op oracle on the same bytes: bf16 outputs bit for bit, the fp32 row sums
within their summation bound; autograd; determinism; the LLM-size row."""
import numpy as np
import pytest
import torch

from mhc_ops_b200 import mhc_post, mhc_post_backward, mhc_post_fn
from oracle import post_oracle as P
from tests._gpu import DEV, bits

pytestmark = pytest.mark.gpu


def _inputs(B, S, n, D, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, S, n, D, generator=g).to(torch.bfloat16)
    y = torch.randn(B, S, D, generator=g).to(torch.bfloat16)
    dout = torch.randn(B, S, n, D, generator=g).to(torch.bfloat16)
    h_res = torch.randn(B, S, n, n, generator=g) * 0.5
    h_post = torch.rand(B, S, n, generator=g) * 2.0
    return x, y, dout, h_res, h_post


def _check(B, S, n, D, seed, sample=None):
    x, y, dout, h_res, h_post = _inputs(B, S, n, D, seed)
    d = [t.to(DEV) for t in (x, y, dout, h_res, h_post)]
    out = mhc_post(d[0], d[3], d[4], d[1])
    dx, dh_res, dh_post, dy = mhc_post_backward(d[0], d[3], d[4], d[1], d[2])
    torch.cuda.synchronize()
    T = B * S
    rows = np.arange(T) if sample is None else np.asarray(sample)
    fl = lambda t, *s: t.reshape(T, *s)[rows]   # noqa: E731
    xb, yb, gb = bits(fl(x, n, D)), bits(fl(y, D)), bits(fl(dout, n, D))
    hr, hp = fl(h_res, n, n).numpy(), fl(h_post, n).numpy()
    ref_out = P.post_forward(xb, hr, hp, yb)
    r_dx, r_dhr, r_dhp, r_dy = P.post_backward(xb, hr, hp, yb, gb)
    tag = f"{B}x{S}x{n}x{D}"
    assert np.array_equal(bits(fl(out.cpu(), n, D)), ref_out), f"{tag} out"
    assert np.array_equal(bits(fl(dx.cpu(), n, D)), r_dx), f"{tag} dx"
    assert np.array_equal(bits(fl(dy.cpu(), D)), r_dy), f"{tag} dy"
    sr, sp = P.post_backward_term_scale(xb, yb, gb)
    bound = (D / 32 + 8) * 2.0 ** -24   # per-lane fp32 sums of D/32 products, then a 5-level tree
    assert (np.abs(fl(dh_res.cpu(), n, n).numpy() - r_dhr) <= bound * sr + 1e-30).all(), f"{tag} dh_res"
    assert (np.abs(fl(dh_post.cpu(), n).numpy() - r_dhp) <= bound * sp + 1e-30).all(), f"{tag} dh_post"


@pytest.mark.parametrize("B,S,n,D", [
    (2, 100, 4, 4096),   # LLM row width, 16-byte vectors
    (1, 70, 8, 512),     # n = 8
    (1, 33, 3, 40),      # odd n, D a multiple of 8
    (1, 17, 2, 36),      # D not a multiple of 8: the scalar kernels
    (3, 5, 1, 8),        # n = 1
])
def test_post_op_vs_oracle(B, S, n, D):
    _check(B, S, n, D, seed=B * 1000 + S * 10 + n)


def test_post_op_llm_size_sampled_rows():
    """B=4,S=4096,n=4,D=4096 on the GPU; 64 sampled tokens checked against the oracle."""
    rng = np.random.default_rng(5)
    _check(4, 4096, 4, 4096, seed=77, sample=np.sort(rng.choice(4 * 4096, 64, replace=False)))


def test_post_op_zero_tokens_and_determinism():
    x, y, dout, h_res, h_post = [t.to(DEV) for t in _inputs(1, 0, 4, 64, 1)]
    assert mhc_post(x, h_res, h_post, y).shape == (1, 0, 4, 64)
    x, y, dout, h_res, h_post = [t.to(DEV) for t in _inputs(2, 300, 4, 1024, 2)]
    a = mhc_post_backward(x, h_res, h_post, y, dout)
    b = mhc_post_backward(x, h_res, h_post, y, dout)
    torch.cuda.synchronize()
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_post_op_autograd_matches_backward():
    x, y, dout, h_res, h_post = [t.to(DEV) for t in _inputs(1, 64, 4, 256, 3)]
    xs, ys = x.clone().requires_grad_(), y.clone().requires_grad_()
    hr, hp = h_res.clone().requires_grad_(), h_post.clone().requires_grad_()
    out = mhc_post_fn(xs, hr, hp, ys)
    out.backward(dout)
    dx, dh_res, dh_post, dy = mhc_post_backward(x, h_res, h_post, y, dout)
    torch.cuda.synchronize()
    assert torch.equal(xs.grad, dx) and torch.equal(ys.grad, dy)
    assert torch.equal(hr.grad, dh_res) and torch.equal(hp.grad, dh_post)
