"""The TORCH_LIBRARY(mhc, ...) operators on the CPU: the library registers
torch.ops.mhc.fwd / bwd with their schemas, the Meta kernels give the output
shapes and dtypes of the reference's golden functions
(src/forward/golden.py:65-69, src/backward/golden.py:96, dgamma flat [nD])
without a device, and CPU tensors have no kernel (no CPU fallback)."""
import pytest
import torch

from mhc_ops_b200 import ops


def _meta_inputs(B=2, S=8, n=4, D=64):
    N = n * n + 2 * n
    m = dict(device="meta")
    return dict(x=torch.empty(B, S, n, D, dtype=torch.bfloat16, **m), phi=torch.empty(N, n * D, **m),
                alpha=torch.empty(3, **m), bias=torch.empty(N, **m), inv_rms=torch.empty(B, S, **m),
                h_mix=torch.empty(B, S, N, **m), h_pre=torch.empty(B, S, n, **m), h_post=torch.empty(B, S, n, **m),
                dh_in=torch.empty(B, S, D, dtype=torch.bfloat16, **m), dh_post=torch.empty(B, S, n, **m),
                dh_res=torch.empty(B, S, n, n, **m), gamma=torch.empty(n, D, **m))


def test_operators_are_registered_with_their_schemas():
    ops.load()
    fwd = str(torch.ops.mhc.fwd.default._schema)
    bwd = str(torch.ops.mhc.bwd.default._schema)
    assert fwd.startswith("mhc::fwd(Tensor x, Tensor phi, Tensor alpha, Tensor bias, float norm_eps=")
    assert "Tensor? gamma" in bwd and bwd.startswith("mhc::bwd(Tensor x, Tensor phi, Tensor alpha, Tensor inv_rms")


@pytest.mark.parametrize("n,D", [(4, 64), (8, 128), (2, 40)])
def test_meta_kernels_give_the_golden_output_shapes(n, D):
    t = _meta_inputs(n=n, D=D)
    B, S, N = 2, 8, n * n + 2 * n
    out = ops.fwd(t["x"], t["phi"], t["alpha"], t["bias"])
    want = [((B, S, D), torch.bfloat16), ((B, S, n), torch.float32), ((B, S, n, n), torch.float32),
            ((B, S), torch.float32), ((B, S, N), torch.float32), ((B, S, n), torch.float32)]
    assert [(tuple(o.shape), o.dtype) for o in out] == want
    for g in (t["gamma"], None):
        out = ops.bwd(t["x"], t["phi"], t["alpha"], t["inv_rms"], t["h_mix"], t["h_pre"], t["h_post"], t["dh_in"],
                      t["dh_post"], t["dh_res"], g)
        want = [((B, S, n, D), torch.bfloat16), ((N, n * D), torch.float32), ((3,), torch.float32),
                ((N,), torch.float32), ((n * D,), torch.float32)]
        assert [(tuple(o.shape), o.dtype) for o in out] == want


def test_cpu_tensors_have_no_kernel():
    t = {k: torch.zeros(v.shape, dtype=v.dtype) for k, v in _meta_inputs().items()}
    with pytest.raises((NotImplementedError, RuntimeError)):
        ops.fwd(t["x"], t["phi"], t["alpha"], t["bias"])
