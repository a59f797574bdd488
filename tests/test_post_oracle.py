"""The post-op oracle (x_next = h_res x + h_post y and its gradient) against an
independent derivation: torch autograd in float64 on the CPU.  The reference
has no post-op, so this is what the oracle is checked against."""
import numpy as np
import pytest
import torch

from oracle import mhc_oracle as O
from oracle import post_oracle as P


def _case(T, n, D, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, n, D, generator=g).to(torch.bfloat16)
    y = torch.randn(T, D, generator=g).to(torch.bfloat16)
    dout = torch.randn(T, n, D, generator=g).to(torch.bfloat16)
    h_res = torch.randn(T, n, n, generator=g) * 0.5
    h_post = torch.rand(T, n, generator=g) * 2.0
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)   # noqa: E731
    return x, y, dout, h_res, h_post, bits


def _ulp_close(ours_u16, ref64, ulps=1.0):
    """bf16 result within `ulps` bf16 ulp of the float64 value (plus an fp32-order floor)."""
    ours = O.bf16_to_f32(ours_u16).astype(np.float64)
    ulp = O.bf16_ulp(ref64.astype(np.float32)).astype(np.float64)
    return np.abs(ours - ref64) <= ulps * ulp + 2.0 ** -20 * np.abs(ref64) + 1e-30


@pytest.mark.parametrize("T,n,D", [(7, 4, 64), (5, 8, 40), (3, 1, 16), (4, 3, 24)])
def test_post_oracle_matches_float64_autograd(T, n, D):
    x, y, dout, h_res, h_post, bits = _case(T, n, D, seed=T * 100 + n)
    xd = x.double().requires_grad_()
    yd = y.double().requires_grad_()
    hr = h_res.double().requires_grad_()
    hp = h_post.double().requires_grad_()
    out64 = torch.einsum("tij,tjd->tid", hr, xd) + hp[:, :, None] * yd[:, None, :]
    out64.backward(dout.double())

    out = P.post_forward(bits(x), h_res.numpy(), h_post.numpy(), bits(y))
    assert _ulp_close(out, out64.detach().numpy()).all()
    dx, dh_res, dh_post, dy = P.post_backward(bits(x), h_res.numpy(), h_post.numpy(), bits(y), bits(dout))
    assert _ulp_close(dx, xd.grad.numpy()).all()
    assert _ulp_close(dy, yd.grad.numpy()).all()
    sr, sp = P.post_backward_term_scale(bits(x), bits(y), bits(dout))
    assert (np.abs(dh_res - hr.grad.numpy()) <= 2.0 ** -23 * sr + 1e-30).all()
    assert (np.abs(dh_post - hp.grad.numpy()) <= 2.0 ** -23 * sp + 1e-30).all()


def test_post_oracle_bf16_outputs_follow_the_stated_order():
    """The bf16 outputs are the float32 ascending-order sums, rounded once."""
    x, y, dout, h_res, h_post, bits = _case(6, 4, 32, seed=9)
    xf, yf = x.float().numpy(), y.float().numpy()
    hr, hp = h_res.numpy(), h_post.numpy()
    acc = hr[:, 2, 0:1] * xf[:, 0]
    for j in range(1, 4):
        acc = acc + hr[:, 2, j:j + 1] * xf[:, j]
    acc = acc + hp[:, 2:3] * yf
    out = P.post_forward(bits(x), hr, hp, bits(y))
    assert np.array_equal(out[:, 2], O.f32_to_bf16(acc))


def test_post_op_cpu_tensors_raise():
    from mhc_ops_b200 import mhc_post
    x, y, dout, h_res, h_post, _ = _case(2, 4, 16, seed=1)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        mhc_post(x.reshape(1, 2, 4, 16), h_res.reshape(1, 2, 4, 4), h_post.reshape(1, 2, 4), y.reshape(1, 2, 16))
