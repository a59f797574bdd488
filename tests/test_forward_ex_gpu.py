"""The forward's options (mhc_fwd_ex): a bf16 phi and the next sublayer's
RMSNorm statistic of h_in.

* bf16 phi is exact in one bf16 term: the forward must give the same outputs,
  bit for bit, as the fp32-phi forward given the same values widened to fp32
  (whose second and third split terms are then zero), and match the oracle;
* h_in_rstd = 1 / sqrt(mean_d(h_in^2) + eps) over the bf16 h_in row: checked
  against that formula evaluated in float64 on the returned h_in, and h_in
  itself is bit for bit the one mhc_forward_pre returns.
"""
import numpy as np
import pytest
import torch

from mhc_ops_b200 import mhc_forward_pre, mhc_forward_pre_fused_norm
from mhc_ops_b200.synthetic import make_inputs
from oracle import mhc_oracle as O
from tests._gpu import DEV, assert_fwd_close, bits

pytestmark = pytest.mark.gpu

SHAPES = [(4, 1024, 4, 4096),   # fused tensor-core forward
          (1, 300, 8, 1024),    # n = 8: projection + row kernel
          (1, 50, 3, 24),       # generic kernels (bf16 phi widened into the workspace)
          (1, 130, 4, 64)]      # ragged last tile


@pytest.mark.parametrize("B,S,n,D", SHAPES)
def test_bf16_phi_equals_fp32_phi_of_the_same_values(B, S, n, D):
    inp = make_inputs(B, S, n, D, seed=41)
    d = inp.to(DEV)
    phi_bf16 = d.phi.to(torch.bfloat16)
    a = mhc_forward_pre(d.x, phi_bf16, d.alpha, d.bias, outflag=True)
    b = mhc_forward_pre(d.x, phi_bf16.float(), d.alpha, d.bias, outflag=True)
    torch.cuda.synchronize()
    for i, (u, v) in enumerate(zip(a, b)):
        assert torch.equal(u, v), f"output {i}: bf16 phi differs from the same phi in fp32"
    if B * S <= 1024:
        xb = bits(inp.x)
        ref = O.forward(xb, phi_bf16.float().cpu().numpy(), inp.alpha.numpy(), inp.bias.numpy(), outflag=True)
        assert_fwd_close(a, ref, xb, tag=f"bf16 phi {B}x{S}x{n}x{D}")


@pytest.mark.parametrize("B,S,n,D", SHAPES)
def test_h_in_rstd_is_the_rmsnorm_factor_of_h_in(B, S, n, D):
    d = make_inputs(B, S, n, D, seed=42).to(DEV)
    eps = 1e-5
    h_in, rstd, h_post, h_res = mhc_forward_pre_fused_norm(d.x, d.phi, d.alpha, d.bias, h_in_norm_eps=eps)
    plain = mhc_forward_pre(d.x, d.phi, d.alpha, d.bias)
    torch.cuda.synchronize()
    assert torch.equal(h_in, plain[0]) and torch.equal(h_post, plain[1]) and torch.equal(h_res, plain[2])
    want = 1.0 / torch.sqrt(h_in.double().square().mean(-1) + eps)
    err = ((rstd.double() - want).abs() / want).max().item()
    assert err <= 1e-5, f"h_in_rstd rel err {err:.3g}"
    assert rstd.shape == (B, S) and np.isfinite(rstd.cpu().numpy()).all()


@pytest.mark.parametrize("B,S,n,D", [(4, 1024, 4, 4096), (1, 300, 8, 1024), (1, 130, 4, 64), (2, 64, 4, 256)])
@pytest.mark.parametrize("bf16_phi", [False, True])
def test_fp8_x_forward_equals_bf16_forward_on_the_dequantized_x(B, S, n, D, bf16_phi):
    """x as e4m3 with a power-of-two scale per token: x8 * 2^e is exact in
    bf16, and the fp8 forward must give, bit for bit, the outputs of the bf16
    forward on that x (and so match the oracle on it)."""
    from mhc_ops_b200 import mhc_forward_pre_fp8, quantize_fp8_pow2
    inp = make_inputs(B, S, n, D, seed=43)
    d = inp.to(DEV)
    # spread the per-token magnitudes so the exponents differ from token to token
    x = (d.x.float() * torch.exp2(torch.randint(-6, 7, (B, S, 1, 1), device=DEV).float())).to(torch.bfloat16)
    x8, e = quantize_fp8_pow2(x)
    x_hat = (x8.float() * torch.exp2(e.float())[:, :, None, None]).to(torch.bfloat16)
    assert torch.equal(x_hat.float(), x8.float() * torch.exp2(e.float())[:, :, None, None])   # exact in bf16
    phi = d.phi.to(torch.bfloat16) if bf16_phi else d.phi
    a = mhc_forward_pre_fp8(x8, e, phi, d.alpha, d.bias, outflag=True)
    b = mhc_forward_pre(x_hat, phi, d.alpha, d.bias, outflag=True)
    torch.cuda.synchronize()
    for i, (u, v) in enumerate(zip(a, b)):
        assert torch.equal(u, v), f"output {i}: fp8 forward differs from the bf16 forward on x8 * 2^e"
    if B * S <= 512 and not bf16_phi:
        xb = bits(x_hat)
        ref = O.forward(xb, inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), outflag=True)
        assert_fwd_close(a, ref, xb, tag=f"fp8 x {B}x{S}x{n}x{D}")


def test_fp8_x_forward_refuses_shapes_off_the_tensor_cores():
    from mhc_ops_b200 import _lib, mhc_forward_pre_fp8, quantize_fp8_pow2
    d = make_inputs(1, 20, 3, 24, seed=44).to(DEV)
    x8, e = quantize_fp8_pow2(d.x)
    with pytest.raises(_lib.MhcError):
        mhc_forward_pre_fp8(x8, e, d.phi, d.alpha, d.bias)


@pytest.mark.parametrize("B,S,n,D,budget", [(4, 1024, 4, 4096, 140),   # fused forward on 140 of the SMs
                                            (4, 1024, 4, 4096, 37),    # a quarter of them
                                            (1, 300, 8, 1024, 100)])   # projection + row kernel
def test_sm_budget_gives_the_same_bits(B, S, n, D, budget):
    """sm_budget (the data-parallel bench leaves that many SMs to the NCCL
    all-reduce) only shrinks the grids: every output equals, bit for bit, the
    forward on every SM."""
    inp = make_inputs(B, S, n, D, seed=43)
    d = inp.to(DEV)
    a = mhc_forward_pre(d.x, d.phi, d.alpha, d.bias, outflag=True)
    b = mhc_forward_pre(d.x, d.phi, d.alpha, d.bias, outflag=True, sm_budget=budget)
    torch.cuda.synchronize()
    for i, (u, v) in enumerate(zip(a, b)):
        assert torch.equal(u, v), f"output {i}: sm_budget={budget} differs from the full grid"
