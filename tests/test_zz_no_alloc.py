"""mhc_fwd_static: the forward entry point that allocates nothing.

Some callers of this library cannot call cudaMalloc: a host whose own
allocator owns all device memory, or a serving runtime that plans memory ahead
and forbids allocation while it runs.  mhc_fwd_static serves them by taking its
scratch from a fixed 16 MiB device array inside the library instead of a
caller workspace.  These tests call it through the C ABI, as such a caller
would, and check it against mhc_fwd with a caller workspace.  The file is
collected last so that a failure here comes after every other test has run.
"""
import ctypes

import numpy as np
import pytest
import torch

from mhc_ops_b200 import _lib
from mhc_ops_b200.synthetic import make_inputs

MHC_ERR_LIMIT = 8
FP32_TOL = 1e-4   # fp32 outputs: max|a-b| / max|ref|, as in the other GPU tests


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


def _bf16_ulps_apart(a, b):
    """Distance in bf16 ulps between two bf16 tensors of finite values (same sign or zero)."""
    ia = a.view(torch.int16).to(torch.int32)
    ib = b.view(torch.int16).to(torch.int32)
    # map the sign-magnitude bit pattern onto a monotone integer line
    ia = torch.where(ia < 0, -(ia & 0x7FFF), ia)
    ib = torch.where(ib < 0, -(ib & 0x7FFF), ib)
    return (ia - ib).abs().max().item() if a.numel() else 0


@pytest.mark.gpu
def test_static_forward_matches_workspace_forward_two_calls_in_a_row():
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    # Two calls in a row on the same array, with different shapes so that the
    # second call reads its scratch over what the first one left there.
    for B, S, n, D, seed in ((1, 300, 4, 4096, 11), (2, 100, 8, 1024, 12)):
        T = B * S
        d = make_inputs(B, S, n, D, seed=seed).to("cuda")
        mine = _outputs(T, n, D)
        assert lib.mhc_fwd_static(ctypes.byref(_args(d, mine, T, n, D)), stream) == 0

        size = ctypes.c_size_t(0)
        assert lib.mhc_fwd_workspace_size(T, n, D, ctypes.byref(size)) == 0
        ws = torch.zeros(size.value, dtype=torch.uint8, device="cuda")
        ref = _outputs(T, n, D)
        assert lib.mhc_fwd(ctypes.byref(_args(d, ref, T, n, D, ws)), stream) == 0
        torch.cuda.synchronize()

        for name, o, r in zip(("h_post", "h_res", "inv_rms", "h_mix", "h_pre"), mine[1:], ref[1:]):
            err = ((o - r).abs().max() / r.abs().max().clamp_min(1e-30)).item()
            assert err <= FP32_TOL, f"n={n} D={D} {name}: rel err {err:.3g}"
        assert _bf16_ulps_apart(mine[0], ref[0]) <= 1, f"n={n} D={D} h_in differs by more than one bf16 ulp"
        assert np.isfinite(mine[0].float().cpu().numpy()).all()


def test_static_forward_rejects_shapes_beyond_its_array():
    """Shapes whose split-phi images exceed 16 MiB are refused before any device work."""
    lib = _lib.load()
    a = _lib.FwdArgs(tokens=1, n=8, D=6592, norm_eps=1e-6, hc_eps=1e-6)
    assert lib.mhc_fwd_static(ctypes.byref(a), None) == MHC_ERR_LIMIT
    a = _lib.FwdArgs(tokens=1, n=4, D=26240, norm_eps=1e-6, hc_eps=1e-6)
    assert lib.mhc_fwd_static(ctypes.byref(a), None) == MHC_ERR_LIMIT
    assert b"limit" in lib.mhc_status_string(MHC_ERR_LIMIT)
