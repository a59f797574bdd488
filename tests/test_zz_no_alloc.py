"""mhc_fwd_static: the forward entry point that allocates nothing.

Some callers of this library cannot call cudaMalloc: a host whose own
allocator owns all device memory, or a serving runtime that plans memory ahead
and forbids allocation while it runs.  mhc_fwd_static serves them by taking its
scratch from a fixed 16 MiB device array inside the library instead of a
caller workspace.  These tests call it through the C ABI, as such a caller
would, and check it against mhc_fwd with a caller workspace (bit for bit)
and against the CPU oracle.  The file is collected last so that a failure
here comes after every other test has run.
"""
import ctypes

import pytest
import torch

from mhc_ops_b200 import _lib
from mhc_ops_b200.synthetic import make_inputs
from oracle import mhc_oracle as O
from tests._gpu import assert_fwd_close, bits

MHC_ERR_LIMIT = 8


def _outputs(T, n, D):
    N = n * n + 2 * n
    return (torch.empty(T, D, dtype=torch.bfloat16, device="cuda"), torch.empty(T, n, device="cuda"),
            torch.empty(T, n, n, device="cuda"), torch.empty(T, device="cuda"), torch.empty(T, N, device="cuda"),
            torch.empty(T, n, device="cuda"))


def _args(d, outs, T, n, D, ws=None):
    return _lib.FwdArgs(x=d.x.data_ptr(), phi=d.phi.data_ptr(), alpha=d.alpha.data_ptr(), bias=d.bias.data_ptr(),
                        h_in=outs[0].data_ptr(), h_post=outs[1].data_ptr(), h_res=outs[2].data_ptr(),
                        inv_rms=outs[3].data_ptr(), h_mix=outs[4].data_ptr(), h_pre=outs[5].data_ptr(),
                        tokens=T, n=n, D=D, norm_eps=1e-6, hc_eps=1e-6,
                        workspace=None if ws is None else ws.data_ptr(),
                        workspace_bytes=0 if ws is None else ws.numel())


@pytest.mark.gpu
def test_static_forward_matches_workspace_forward_two_calls_in_a_row():
    """Two n=4 calls in a row (the fused forward, whose per-tile counters live
    in the scratch): the first, larger call leaves its counters at nonzero
    values, so the second call must clear what it needs.  A third call takes
    the n=8 two-kernel form.  Each must match mhc_fwd with a caller workspace
    bit for bit (same kernels, same plan) and the oracle within the tolerance
    of the other GPU tests."""
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for B, S, n, D, seed in ((1, 600, 4, 4096, 11), (1, 300, 4, 4096, 12), (2, 100, 8, 1024, 13)):
        T = B * S
        inp = make_inputs(B, S, n, D, seed=seed)
        d = inp.to("cuda")
        mine = _outputs(T, n, D)
        assert lib.mhc_fwd_static(ctypes.byref(_args(d, mine, T, n, D)), stream) == 0

        size = ctypes.c_size_t(0)
        assert lib.mhc_fwd_workspace_size(T, n, D, ctypes.byref(size)) == 0
        ws = torch.zeros(size.value, dtype=torch.uint8, device="cuda")
        ref = _outputs(T, n, D)
        assert lib.mhc_fwd(ctypes.byref(_args(d, ref, T, n, D, ws)), stream) == 0
        torch.cuda.synchronize()

        for name, o, r in zip(("h_in", "h_post", "h_res", "inv_rms", "h_mix", "h_pre"), mine, ref):
            assert torch.equal(o, r), f"n={n} D={D} T={T} {name}: mhc_fwd_static differs from mhc_fwd"

        # and against the CPU oracle, as every forward test checks it
        xb = bits(inp.x)
        oracle = O.forward(xb, inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), outflag=True)
        shaped = (mine[0].reshape(B, S, D), mine[1].reshape(B, S, n), mine[2].reshape(B, S, n, n),
                  mine[3].reshape(B, S), mine[4].reshape(B, S, -1), mine[5].reshape(B, S, n))
        assert_fwd_close(shaped, oracle, xb, tag=f"static {B}x{S}x{n}x{D}")


def test_static_forward_rejects_shapes_beyond_its_array():
    """Shapes whose split-phi images exceed 16 MiB are refused before any device work."""
    lib = _lib.load()
    a = _lib.FwdArgs(tokens=1, n=8, D=6592, norm_eps=1e-6, hc_eps=1e-6)
    assert lib.mhc_fwd_static(ctypes.byref(a), None) == MHC_ERR_LIMIT
    a = _lib.FwdArgs(tokens=1, n=4, D=26240, norm_eps=1e-6, hc_eps=1e-6)
    assert lib.mhc_fwd_static(ctypes.byref(a), None) == MHC_ERR_LIMIT
    assert b"limit" in lib.mhc_status_string(MHC_ERR_LIMIT)
