"""MHCPreFunction (autograd) against a plain PyTorch fp64 reference of the same op."""
import pytest
import torch

from mhc_ops_b200 import mhc_pre
from mhc_ops_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu


def _torch_reference(x, phi, alpha, bias, gamma, eps=1e-6):
    B, S, n, D = x.shape
    vec = x.reshape(B, S, n * D)
    w = phi if gamma is None else phi * gamma.reshape(1, -1)
    h_mix = vec @ w.t()
    ir = torch.rsqrt(vec.square().mean(-1, keepdim=True) + eps)
    t = h_mix * ir
    h_pre = torch.sigmoid(alpha[0] * t[..., :n] + bias[:n]) + eps
    h_post = 2 * torch.sigmoid(alpha[1] * t[..., n:2 * n] + bias[n:2 * n])
    h_res = alpha[2] * t[..., 2 * n:].reshape(B, S, n, n) + bias[2 * n:].view(n, n)
    h_in = (h_pre.unsqueeze(-1) * x).sum(2)
    return h_in, h_post, h_res


@pytest.mark.parametrize("use_gamma", [True, False])
@pytest.mark.parametrize("n,D", [(4, 256), (8, 128)])
def test_autograd_matches_fp64_torch(use_gamma, n, D):
    inp = make_inputs(2, 48, n, D, seed=21).to("cuda")
    leaves = {k: getattr(inp, k).clone().requires_grad_(True) for k in ("phi", "alpha", "bias", "gamma")}
    x = inp.x.clone().requires_grad_(True)
    gamma = leaves["gamma"] if use_gamma else None
    h_in, h_post, h_res = mhc_pre(x, leaves["phi"], leaves["alpha"], leaves["bias"], gamma)
    loss = (h_in.float() * inp.dh_in.float()).sum() + (h_post * inp.dh_post).sum() + (h_res * inp.dh_res).sum()
    loss.backward()

    ref_leaves = {k: getattr(inp, k).double().clone().requires_grad_(True) for k in ("phi", "alpha", "bias", "gamma")}
    xr = inp.x.double().clone().requires_grad_(True)
    rg = ref_leaves["gamma"] if use_gamma else None
    r_in, r_post, r_res = _torch_reference(xr, ref_leaves["phi"], ref_leaves["alpha"], ref_leaves["bias"], rg)
    rloss = (r_in * inp.dh_in.double()).sum() + (r_post * inp.dh_post.double()).sum() + (r_res * inp.dh_res.double()).sum()
    rloss.backward()

    def rel(a, b):
        return ((a.double() - b).abs().max() / b.abs().max()).item()

    assert rel(h_post, r_post) < 1e-4 and rel(h_res, r_res) < 1e-4
    assert rel(h_in.float(), r_in) < 1e-2
    for k in ("phi", "alpha", "bias") + (("gamma",) if use_gamma else ()):
        assert rel(leaves[k].grad, ref_leaves[k].grad) < 1e-4, k
    assert rel(x.grad.float(), xr.grad) < 1e-2
    if not use_gamma:
        assert leaves["gamma"].grad is None


def test_torch_compile_of_mhc_pre_matches_eager_bit_for_bit():
    """mhc_pre under torch.compile: dynamo traces the registered operators
    (torch.ops.mhc.fwd / bwd, Meta kernels for the shapes) as graph nodes; the
    compiled forward and backward run the same kernels and must give the
    eager results bit for bit."""
    inp = make_inputs(2, 64, 4, 256, seed=23).to("cuda")

    def run(fn):
        leaves = {k: getattr(inp, k).clone().requires_grad_(True) for k in ("phi", "alpha", "bias", "gamma")}
        x = inp.x.clone().requires_grad_(True)
        h_in, h_post, h_res = fn(x, leaves["phi"], leaves["alpha"], leaves["bias"], leaves["gamma"])
        loss = (h_in.float() * inp.dh_in.float()).sum() + (h_post * inp.dh_post).sum() + (h_res * inp.dh_res).sum()
        loss.backward()
        return (h_in, h_post, h_res, x.grad) + tuple(leaves[k].grad for k in ("phi", "alpha", "bias", "gamma"))

    eager = run(mhc_pre)
    compiled = run(torch.compile(mhc_pre, fullgraph=True))
    for i, (a, b) in enumerate(zip(eager, compiled)):
        assert torch.equal(a, b), f"output {i} differs under torch.compile"
