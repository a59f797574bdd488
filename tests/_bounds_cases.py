"""The cases the debug-bounds test runs twice: in a child process on the
-DMHC_DEBUG_BOUNDS library (MHC_OPS_LIBRARY set), where the record of
out-of-buffer accesses must stay empty after every call, and in the test
process on the normal library.  Odd shapes on purpose (a bounds diagnostic
is only as good as the edges it visits): one token, prime token counts, D
not a multiple of 8, n = 2, 3, 4, 5, 8, every forward option, both backward
forms, the post-op and the static forward.

    python -m tests._bounds_cases OUT.npz     (child: writes every output)
"""
from __future__ import annotations

import ctypes
import sys

import numpy as np
import torch

from mhc_ops_b200 import _lib
from mhc_ops_b200.backward import mhc_backward_manual
from mhc_ops_b200.forward import (mhc_forward_pre, mhc_forward_pre_fp8, mhc_forward_pre_fused_norm,
                                  quantize_fp8_pow2)
from mhc_ops_b200.post import mhc_post, mhc_post_backward
from mhc_ops_b200.synthetic import make_inputs

# (B, S, n, D): which kernels they reach
SHAPES = (
    (1, 1, 4, 64),      # one token: tensor-core forward and backward
    (1, 131, 4, 4096),  # prime token count: fused forward, n = 4 tensor-core backward
    (1, 257, 3, 100),   # D not a multiple of 8: generic kernels
    (1, 97, 8, 1024),   # n = 8: two-kernel forward, tiled backward
    (2, 7, 2, 24),      # n = 2, tiny
    (1, 130, 5, 128),   # n = 5: tiled backward on the CUDA cores
)


def _arr(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float8_e4m3fn):
        return t.view(torch.uint8).numpy().copy()
    return t.numpy().copy()


def _check_record(where: str, debug: bool) -> None:
    if debug:
        rec = _lib.debug_bounds(clear=True, raise_on_hit=False)
        assert rec["count"] == 0, f"{where}: access outside the call's buffers {rec}"


def _static_forward(d, T, n, D):
    N = n * n + 2 * n
    outs = (torch.empty(T, D, dtype=torch.bfloat16, device="cuda"), torch.empty(T, n, device="cuda"),
            torch.empty(T, n, n, device="cuda"), torch.empty(T, device="cuda"), torch.empty(T, N, device="cuda"),
            torch.empty(T, n, device="cuda"))
    a = _lib.FwdArgs(x=d.x.data_ptr(), phi=d.phi.data_ptr(), alpha=d.alpha.data_ptr(), bias=d.bias.data_ptr(),
                     h_in=outs[0].data_ptr(), h_post=outs[1].data_ptr(), h_res=outs[2].data_ptr(),
                     inv_rms=outs[3].data_ptr(), h_mix=outs[4].data_ptr(), h_pre=outs[5].data_ptr(),
                     tokens=T, n=n, D=D, norm_eps=1e-6, hc_eps=1e-6)
    st = _lib.load().mhc_fwd_static(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "mhc_fwd_static")
    return outs


def run_cases(debug: bool) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}

    def keep(tag, tensors):
        for i, t in enumerate(tensors):
            out[f"{tag}/{i}"] = _arr(t)

    for si, (B, S, n, D) in enumerate(SHAPES):
        tag = f"{B}x{S}x{n}x{D}"
        d = make_inputs(B, S, n, D, seed=40 + si).to("cuda")
        fw = mhc_forward_pre(d.x, d.phi, d.alpha, d.bias, outflag=True)
        torch.cuda.synchronize()
        _check_record(f"{tag} forward", debug)
        keep(f"{tag}/fwd", fw)
        bw = mhc_backward_manual(d.x, d.phi, d.alpha, d.bias, fw[3], fw[4], fw[5], fw[1], d.dh_in, d.dh_post,
                                 d.dh_res, d.gamma)
        torch.cuda.synchronize()
        _check_record(f"{tag} backward", debug)
        keep(f"{tag}/bwd", bw)
        rc = mhc_backward_manual(d.x, d.phi, d.alpha, d.bias, None, None, None, fw[1], d.dh_in, d.dh_post,
                                 d.dh_res, d.gamma)
        torch.cuda.synchronize()
        _check_record(f"{tag} backward (recompute)", debug)
        keep(f"{tag}/bwd_rc", rc)
        fn = mhc_forward_pre_fused_norm(d.x, d.phi.bfloat16(), d.alpha, d.bias, outflag=True)
        torch.cuda.synchronize()
        _check_record(f"{tag} forward (bf16 phi, h_in_rstd)", debug)
        keep(f"{tag}/fwd_ex", fn)
        if n in (4, 8) and D % 64 == 0:
            x8, xe = quantize_fp8_pow2(d.x)
            f8 = mhc_forward_pre_fp8(x8, xe, d.phi, d.alpha, d.bias, outflag=True)
            torch.cuda.synchronize()
            _check_record(f"{tag} forward (fp8 x)", debug)
            keep(f"{tag}/fwd_fp8", f8)
        y = fw[0]
        po = mhc_post(d.x, fw[2], fw[1], y)
        pb = mhc_post_backward(d.x, fw[2], fw[1], y, po)
        torch.cuda.synchronize()
        _check_record(f"{tag} post-op", debug)
        keep(f"{tag}/post", (po,) + tuple(pb))
        if D % 64 == 0:
            st = _static_forward(d, B * S, n, D)
            torch.cuda.synchronize()
            _check_record(f"{tag} static forward", debug)
            keep(f"{tag}/fwd_static", st)
    return out


def selftest_record() -> dict:
    """The record after mhc_debug_bounds_selftest: one failed check, nothing accessed."""
    ws = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    _lib.debug_bounds(clear=True)
    st = _lib.load().mhc_debug_bounds_selftest(ctypes.c_void_p(ws.data_ptr()),
                                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(st, "mhc_debug_bounds_selftest")
    rec = _lib.debug_bounds(clear=True, raise_on_hit=False)
    rec["workspace"] = ws.data_ptr()
    return rec


def main(path: str) -> None:
    rec = selftest_record()
    out = run_cases(debug=True)
    out["selftest"] = np.array([rec["count"], rec["site"], rec["address"] - rec["workspace"], rec["bytes"]],
                               dtype=np.int64)
    np.savez(path, **out)


if __name__ == "__main__":
    main(sys.argv[1])
