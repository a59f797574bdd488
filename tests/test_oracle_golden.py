"""The CPU oracle (oracle/mhc_oracle.py) against the reference golden fixtures.

Every fixture in tests/golden/ was produced by running the reference's own
golden forward (src/forward/golden.py) and backward (src/backward/golden.py)
on seeded inputs (tests/golden/make_golden.py).  This pins the oracle before
the CUDA path is compared with it.
"""
import warnings

import numpy as np
import pytest

from oracle import mhc_oracle as O
from tests._golden import fixture_names, load_fixture, rel_err

FP32_TOL = 1e-4   # fp32 outputs: max|a-b| / max|ref|  (the stated bar)


@pytest.mark.parametrize("name", fixture_names())
def test_forward_matches_reference_golden(name):
    z = load_fixture(name)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", RuntimeWarning)   # exp overflow inside sigmoid saturates correctly
        h_in, h_post, h_res, inv_rms, h_mix, h_pre = O.forward(z["x"], z["phi"], z["alpha"], z["bias"],
                                                               outflag=True)
    for nm, v in (("h_post", h_post), ("h_res", h_res), ("inv_rms", inv_rms), ("h_mix", h_mix),
                  ("h_pre", h_pre)):
        assert v.shape == z[nm].shape
        assert rel_err(v, z[nm]) <= FP32_TOL, nm
    ok, worst, nbad = O.bf16_within(h_in, z["h_in"], O.forward_term_scale(z["x"], z["h_pre"]))
    assert ok, f"h_in: {nbad} elements beyond 1 ulp (+fp32 floor); worst {worst} ulps"


@pytest.mark.parametrize("name", fixture_names())
def test_backward_matches_reference_golden(name):
    z = load_fixture(name)
    args = (z["x"], z["phi"], z["alpha"], z["bias"], z["inv_rms"], z["h_mix"], z["h_pre"], z["h_post"],
            z["dh_in"], z["dh_post"], z["dh_res"], z["gamma"])
    dx, dphi, dalpha, dbias, dgamma = O.backward(*args)
    for nm, v in (("dphi", dphi), ("dalpha", dalpha), ("dbias", dbias), ("dgamma", dgamma)):
        assert v.shape == z[nm].shape, nm
        assert rel_err(v, z[nm]) <= FP32_TOL, nm
    B, S, n, D = z["shape"]
    assert dgamma.shape == (n * D,)   # flat, golden.py:93
    scale = O.backward_term_scale(z["x"], z["phi"], z["alpha"], z["inv_rms"], z["h_mix"], z["h_pre"],
                                  z["h_post"], z["dh_in"], z["dh_post"], z["dh_res"], z["gamma"])
    ok, worst, nbad = O.bf16_within(dx, z["dx"], scale)
    assert ok, f"dx: {nbad} elements beyond 1 ulp (+fp32 floor); worst {worst} ulps"


def test_bf16_round_trip_and_rne():
    vals = np.array([1.0, -2.5, 3.14159, 1e-30, -0.0, 65504.0, 1.00390625, 1.01171875], np.float32)
    bits = O.f32_to_bf16(vals)
    back = O.bf16_to_f32(bits)
    # 1.00390625 = 1 + 2^-8 is exactly half an ulp above 1.0 -> ties to even -> 1.0
    assert back[6] == 1.0
    # 1.01171875 = 1 + 3*2^-8 -> tie between 1+2^-7 and 1+2^-6 -> even mantissa 1+2^-6
    assert back[7] == np.float32(1.015625)
    assert np.all(O.f32_to_bf16(back) == bits)


def test_gamma_identity_backward_equals_gradient_of_gamma_folded_forward():
    """dphi/dx/dgamma of the golden backward are the gradient of forward(phi * gamma)."""
    torch = pytest.importorskip("torch")
    from mhc_ops_b200.synthetic import make_inputs
    inp = make_inputs(1, 8, 4, 16, seed=5)
    x = inp.x.to(torch.float64).requires_grad_(True)
    phi = inp.phi.double().requires_grad_(True)
    gamma = inp.gamma.double().requires_grad_(True)
    alpha, bias = inp.alpha.double().requires_grad_(True), inp.bias.double().requires_grad_(True)
    B, S, n, D = inp.x.shape
    vec = x.reshape(B, S, n * D)
    h_mix = vec @ (phi * gamma.reshape(1, -1)).t()
    ir = torch.rsqrt(vec.square().mean(-1, keepdim=True) + 1e-6)
    t = h_mix * ir
    h_pre = torch.sigmoid(alpha[0] * t[..., :n] + bias[:n]) + 1e-6
    h_post = 2 * torch.sigmoid(alpha[1] * t[..., n:2 * n] + bias[n:2 * n])
    h_res = alpha[2] * t[..., 2 * n:].reshape(B, S, n, n) + bias[2 * n:].view(n, n)
    h_in = (h_pre.unsqueeze(-1) * x).sum(2)
    loss = ((h_in * inp.dh_in.double()).sum() + (h_post * inp.dh_post.double()).sum()
            + (h_res * inp.dh_res.double()).sum())
    loss.backward()
    # oracle backward with the fp64 forward intermediates rounded to fp32
    xb = inp.x.contiguous().view(torch.int16).numpy().view(np.uint16)
    dx, dphi, dalpha, dbias, dgamma = O.backward(
        xb, inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), ir[..., 0].float().detach().numpy(),
        h_mix.float().detach().numpy(), h_pre.float().detach().numpy(), h_post.float().detach().numpy(),
        inp.dh_in.contiguous().view(torch.int16).numpy().view(np.uint16), inp.dh_post.numpy(),
        inp.dh_res.numpy(), inp.gamma.numpy())
    assert rel_err(dphi, phi.grad.numpy()) < 1e-5
    assert rel_err(dgamma, gamma.grad.reshape(-1).numpy()) < 1e-5
    assert rel_err(dalpha, alpha.grad.numpy()) < 1e-5
    assert rel_err(dbias, bias.grad.numpy()) < 1e-5
    assert rel_err(O.bf16_to_f32(dx), x.grad.numpy()) < 1e-2
