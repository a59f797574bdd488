"""The mHC pre-op as registered torch operators: ``torch.ops.mhc.fwd`` and
``torch.ops.mhc.bwd`` (``TORCH_LIBRARY(mhc, ...)`` in ``csrc/torch_ops.cpp``).

``fwd(x, phi, alpha, bias, norm_eps=1e-6, hc_eps=1e-6)`` returns
``(h_in, h_post, h_res, inv_rms, h_mix, h_pre)``: the reference's
``mhc_forward_pre(..., outflag=True)`` (``src/forward/golden.py:10-69``),
whose Triton call site is ``src/forward/mhc_forward_pre_triton.py:409-417``.

``bwd(x, phi, alpha, inv_rms, h_mix, h_pre, h_post, dh_in, dh_post, dh_res,
gamma, norm_eps=1e-6, hc_eps=1e-6)`` returns ``(dx, dphi, dalpha, dbias,
dgamma)``: the reference's ``mhc_backward_manual``
(``src/backward/golden.py:10-96``), Triton call site
``src/backward/mhc_backward_triton.py:467-473``; ``gamma`` may be None.

The operators run the same kernels as the ctypes API through the C ABI, on the
current CUDA stream, and have Meta kernels, so FakeTensor tracing
(``torch.compile``, ``torch.export``) sees them as single graph nodes.  CPU
tensors fail (there is no CPU kernel).  ``check_status()`` waits for the
device status copies of the operators' workspaces and raises if a kernel's
bounded wait expired in an earlier call.
"""
from __future__ import annotations

import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libmhc_torch.so")
_lock = threading.Lock()
_loaded = False

__all__ = ["load", "fwd", "bwd", "check_status", "lib_path"]


def lib_path() -> str:
    return _LIB_PATH


def load() -> None:
    """Register the ``mhc`` operators (once); raises if the library is not built."""
    global _loaded
    if _loaded:
        return
    with _lock:
        if not _loaded:
            if not os.path.exists(_LIB_PATH):
                raise RuntimeError(f"libmhc_torch.so not found at {_LIB_PATH}; build it with "
                                   "`python -m mhc_ops_b200.build` (there is no fallback)")
            torch.ops.load_library(_LIB_PATH)
            _loaded = True


def fwd(x, phi, alpha, bias, norm_eps: float = 1e-6, hc_eps: float = 1e-6):
    load()
    return torch.ops.mhc.fwd(x, phi, alpha, bias, norm_eps, hc_eps)


def bwd(x, phi, alpha, inv_rms, h_mix, h_pre, h_post, dh_in, dh_post, dh_res, gamma=None,
        norm_eps: float = 1e-6, hc_eps: float = 1e-6):
    load()
    return torch.ops.mhc.bwd(x, phi, alpha, inv_rms, h_mix, h_pre, h_post, dh_in, dh_post, dh_res, gamma,
                             norm_eps, hc_eps)


def check_status() -> None:
    load()
    torch.ops.mhc.check_status()
