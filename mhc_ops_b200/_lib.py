"""ctypes binding of libmhc_ops.so (the C ABI declared in include/mhc_ops.h).

The library is built in-tree (``python -m mhc_ops_b200.build``) and loaded
from ``mhc_ops_b200/lib/libmhc_ops.so``, or from the path in the environment
variable MHC_OPS_LIBRARY (e.g. the debug-bounds build
``lib/libmhc_ops_dbg.so``).  There is no fallback: if the library is missing
or no sm_100 GPU is current, the calls raise.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_PATH = os.environ.get("MHC_OPS_LIBRARY") or os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib",
                                                                "libmhc_ops.so")

MHC_OK = 0
MHC_ERR_DEVICE_TIMEOUT = 6
MHC_ERR_OUT_OF_BOUNDS = 9
MHC_ERR_UNSUPPORTED = 10

_c_void_p = ctypes.c_void_p


class FwdArgs(ctypes.Structure):
    """Mirror of ``mhc_fwd_args`` (include/mhc_ops.h)."""
    _fields_ = [
        ("x", _c_void_p), ("phi", _c_void_p), ("alpha", _c_void_p), ("bias", _c_void_p),
        ("h_in", _c_void_p), ("h_post", _c_void_p), ("h_res", _c_void_p),
        ("inv_rms", _c_void_p), ("h_mix", _c_void_p), ("h_pre", _c_void_p),
        ("tokens", ctypes.c_int64), ("n", ctypes.c_int32), ("D", ctypes.c_int32),
        ("norm_eps", ctypes.c_float), ("hc_eps", ctypes.c_float),
        ("workspace", _c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class FwdExArgs(ctypes.Structure):
    """Mirror of ``mhc_fwd_ex_args`` (include/mhc_ops.h)."""
    _fields_ = [("phi_bf16", _c_void_p), ("h_in_rstd", _c_void_p), ("h_in_eps", ctypes.c_float),
                ("sm_budget", ctypes.c_int32), ("x_fp8", _c_void_p), ("x_exp", _c_void_p)]


class BwdArgs(ctypes.Structure):
    """Mirror of ``mhc_bwd_args`` (include/mhc_ops.h)."""
    _fields_ = [
        ("x", _c_void_p), ("phi", _c_void_p), ("alpha", _c_void_p), ("bias", _c_void_p),
        ("inv_rms", _c_void_p), ("h_mix", _c_void_p), ("h_pre", _c_void_p), ("h_post", _c_void_p),
        ("dh_in", _c_void_p), ("dh_post", _c_void_p), ("dh_res", _c_void_p), ("gamma", _c_void_p),
        ("dx", _c_void_p), ("dphi", _c_void_p), ("dalpha", _c_void_p), ("dbias", _c_void_p),
        ("dgamma", _c_void_p),
        ("tokens", ctypes.c_int64), ("n", ctypes.c_int32), ("D", ctypes.c_int32),
        ("norm_eps", ctypes.c_float), ("hc_eps", ctypes.c_float),
        ("workspace", _c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class PostFwdArgs(ctypes.Structure):
    """Mirror of ``mhc_post_fwd_args`` (include/mhc_ops.h)."""
    _fields_ = [
        ("x", _c_void_p), ("h_res", _c_void_p), ("h_post", _c_void_p), ("y", _c_void_p), ("out", _c_void_p),
        ("tokens", ctypes.c_int64), ("n", ctypes.c_int32), ("D", ctypes.c_int32),
    ]


class PostBwdArgs(ctypes.Structure):
    """Mirror of ``mhc_post_bwd_args`` (include/mhc_ops.h)."""
    _fields_ = [
        ("x", _c_void_p), ("h_res", _c_void_p), ("h_post", _c_void_p), ("y", _c_void_p), ("dout", _c_void_p),
        ("dx", _c_void_p), ("dy", _c_void_p), ("dh_res", _c_void_p), ("dh_post", _c_void_p),
        ("tokens", ctypes.c_int64), ("n", ctypes.c_int32), ("D", ctypes.c_int32),
    ]


# Every symbol include/mhc_ops.h declares, with its ctypes signature.
SIGNATURES = {
    "mhc_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "mhc_last_cuda_error": (ctypes.c_char_p, []),
    "mhc_fwd_workspace_size": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.POINTER(ctypes.c_size_t)]),
    "mhc_fwd": (ctypes.c_int, [ctypes.POINTER(FwdArgs), _c_void_p]),
    "mhc_fwd_static": (ctypes.c_int, [ctypes.POINTER(FwdArgs), _c_void_p]),
    "mhc_fwd_ex_workspace_size": (ctypes.c_int, [ctypes.POINTER(FwdExArgs), ctypes.c_int64, ctypes.c_int32,
                                                 ctypes.c_int32, ctypes.POINTER(ctypes.c_size_t)]),
    "mhc_fwd_ex": (ctypes.c_int, [ctypes.POINTER(FwdArgs), ctypes.POINTER(FwdExArgs), _c_void_p]),
    "mhc_bwd_workspace_size": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.POINTER(ctypes.c_size_t)]),
    "mhc_bwd": (ctypes.c_int, [ctypes.POINTER(BwdArgs), _c_void_p]),
    "mhc_bwd_recompute_workspace_size": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                                        ctypes.POINTER(ctypes.c_size_t)]),
    "mhc_read_device_status": (ctypes.c_int, [_c_void_p, _c_void_p, ctypes.POINTER(ctypes.c_int)]),
    "mhc_selftest_wait_expiry": (ctypes.c_int, [_c_void_p, _c_void_p]),
    "mhc_query_plan": (ctypes.c_int, [ctypes.c_int, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                      ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                      ctypes.POINTER(ctypes.c_int)]),
    "mhc_query_plan_for": (ctypes.c_int, [ctypes.c_int, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                          ctypes.POINTER(ctypes.c_int)]),
    "mhc_query_bwd_grid": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.POINTER(ctypes.c_int32)]),
    "mhc_bwd_workspace_size_for": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.POINTER(ctypes.c_size_t)]),
    "mhc_post_fwd": (ctypes.c_int, [ctypes.POINTER(PostFwdArgs), _c_void_p]),
    "mhc_post_bwd": (ctypes.c_int, [ctypes.POINTER(PostBwdArgs), _c_void_p]),
    "mhc_launch_count": (ctypes.c_uint64, []),
    "mhc_abi_version": (ctypes.c_int, []),
    "mhc_debug_bounds": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint64), ctypes.c_int]),
    "mhc_debug_bounds_selftest": (ctypes.c_int, [_c_void_p, _c_void_p]),
}

_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise RuntimeError(
                    f"libmhc_ops.so not found at {_LIB_PATH}; build it with `python -m mhc_ops_b200.build` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class MhcError(RuntimeError):
    def __init__(self, status: int, where: str):
        lib = load()
        msg = lib.mhc_status_string(status).decode()
        if status == 5:
            msg += f" ({lib.mhc_last_cuda_error().decode()})"
        super().__init__(f"{where}: mhc status {status}: {msg}")
        self.status = status


def check(status: int, where: str) -> None:
    if status != MHC_OK:
        raise MhcError(status, where)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ------------------------------------------------------------------ workspaces
class Workspace:
    """A cached device workspace plus the watch over its device status word.

    The first bytes of every workspace hold the status word that a kernel sets
    to MHC_ERR_DEVICE_TIMEOUT when one of its bounded waits expires (its
    outputs are then invalid).  After each call ``watch`` copies that word into
    pinned host memory on a side stream, ordered after the call's kernels but
    without making the caller's stream wait; the next call through the same
    workspace (``raise_if_timed_out``), or ``check_device_status``, looks at
    the copy and raises ``MhcError(MHC_ERR_DEVICE_TIMEOUT)``.
    """

    def __init__(self, nbytes: int, device: torch.device):
        self.buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        self.device = device
        self.host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.side = torch.cuda.Stream(device=device)
        self.done = None          # event recorded on the side stream after the copy
        self.where = ""

    def watch(self, stream: torch.cuda.Stream, where: str) -> None:
        if torch.cuda.is_current_stream_capturing():
            return                # no host-visible copy inside a graph capture
        self.where = where
        self.side.wait_stream(stream)
        with torch.cuda.stream(self.side):
            self.host.copy_(self.buf[:4].view(torch.int32), non_blocking=True)
            self.done = torch.cuda.Event()
            self.done.record(self.side)

    def raise_if_timed_out(self, wait: bool = False) -> None:
        """Raise if an earlier call through this workspace reported a device
        timeout; the word is cleared first, so the next call starts clean.
        With ``wait`` the copy of the last call is waited for."""
        if self.done is None:
            return
        if wait:
            self.done.synchronize()
        elif not self.done.query():
            return                # the last call has not finished yet: look next time
        self.done = None
        code = int(self.host.item())
        if code != MHC_OK:
            self.buf[:4].zero_()
            self.host.zero_()
            raise MhcError(code, f"{self.where} (an earlier call; its outputs are invalid)")


_ws_cache: dict = {}


def workspace(nbytes: int, device: torch.device, stream: torch.cuda.Stream) -> Workspace:
    """A zero-initialised workspace of >= nbytes, cached per (device, stream).

    New workspaces are zero filled once (the first bytes hold the device
    status word); later calls reuse the buffer, ordered by the stream.  A
    timeout an earlier call on this workspace reported is raised here.  While
    the stream captures a CUDA graph the cached workspace is used as it is
    (one made by an earlier call on the stream; none is created).
    """
    key = (device.index, stream.cuda_stream)
    ws = _ws_cache.get(key)
    if torch.cuda.is_current_stream_capturing():
        # inside a CUDA graph capture nothing may be allocated or synchronised:
        # the workspace must come from a call on this stream before the capture
        if ws is None or ws.buf.numel() < nbytes:
            raise RuntimeError(
                "mhc: no workspace for this stream while it is capturing a CUDA graph; run the same call "
                "once on the capturing stream before the capture (as torch's own warm-up advice says)")
        return ws
    if ws is not None:
        # a workspace about to be replaced reports its last call first
        ws.raise_if_timed_out(wait=ws.buf.numel() < nbytes)
    if ws is None or ws.buf.numel() < nbytes:
        ws = Workspace(nbytes, device)
        _ws_cache[key] = ws
    return ws


def check_device_status(device=None) -> None:
    """Wait for the status copies of every cached workspace on ``device``
    (all devices when None) and raise ``MhcError(MHC_ERR_DEVICE_TIMEOUT)`` if
    any call reported an expired device wait."""
    for (idx, _), ws in list(_ws_cache.items()):
        if device is None or torch.device(device).index in (None, idx):
            ws.raise_if_timed_out(wait=True)


def fwd_workspace_size(tokens: int, n: int, D: int, ex: "FwdExArgs | None" = None) -> int:
    out = ctypes.c_size_t(0)
    if ex is None:
        check(load().mhc_fwd_workspace_size(tokens, n, D, ctypes.byref(out)), "mhc_fwd_workspace_size")
    else:
        check(load().mhc_fwd_ex_workspace_size(ctypes.byref(ex), tokens, n, D, ctypes.byref(out)),
              "mhc_fwd_ex_workspace_size")
    return int(out.value)


def bwd_workspace_size(tokens: int, n: int, D: int, recompute: bool = False) -> int:
    out = ctypes.c_size_t(0)
    if recompute:
        check(load().mhc_bwd_recompute_workspace_size(tokens, n, D, ctypes.byref(out)),
              "mhc_bwd_recompute_workspace_size")
    else:
        check(load().mhc_bwd_workspace_size(tokens, n, D, ctypes.byref(out)), "mhc_bwd_workspace_size")
    return int(out.value)


def query_plan(which: int, tokens: int, n: int, D: int, sms: int | None = None) -> dict:
    """Launch plan for forward (which=0) or backward (1) of this shape on the
    current device, or, with ``sms``, on an sm_100 device with that many SMs
    (computed on the host; no device needed)."""
    path, cs, ncl = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    if sms is None:
        check(load().mhc_query_plan(which, tokens, n, D, ctypes.byref(path), ctypes.byref(cs), ctypes.byref(ncl)),
              "mhc_query_plan")
    else:
        check(load().mhc_query_plan_for(which, tokens, n, D, sms, ctypes.byref(path), ctypes.byref(cs),
                                        ctypes.byref(ncl)), "mhc_query_plan_for")
    if not path.value:
        return {"path": "generic"}
    if which == 0:
        return {"path": "tensor-core-fused" if path.value == 2 else "tensor-core", "k_slices": cs.value,
                "ctas": ncl.value}
    if path.value == 3:
        dx = {2: "tensor-core-stream-pairs", 1: "tensor-core", 0: "cuda-cores"}[ncl.value]
        return {"path": "tiled", "token_groups": cs.value, "dx": dx}
    g = (ctypes.c_int32 * 6)()
    check(load().mhc_query_bwd_grid(tokens, n, D, 0 if sms is None else sms, g), "mhc_query_bwd_grid")
    return {"path": "tensor-core", "d_slices": cs.value, "token_groups": ncl.value, "leftover_ctas": g[4],
            "leftover_tiles": g[5], "ctas": g[1] * g[2] + g[4]}


def launch_count() -> int:
    return int(load().mhc_launch_count())


def debug_bounds(clear: bool = True, raise_on_hit: bool = True) -> dict:
    """The debug-bounds record of the calls since the last clear (synchronizes
    the device): ``{"count", "site", "address", "bytes"}``, site = file id *
    100000 + source line of the failed check.  Raises MhcError when an access
    fell outside its call's buffers (unless ``raise_on_hit`` is False), and
    MhcError(MHC_ERR_UNSUPPORTED) with a normal build loaded."""
    rec = (ctypes.c_uint64 * 4)()
    st = load().mhc_debug_bounds(rec, 1 if clear else 0)
    out = {"count": int(rec[0]), "site": int(rec[1]), "address": int(rec[2]), "bytes": int(rec[3])}
    if st == MHC_ERR_OUT_OF_BOUNDS and not raise_on_hit:
        return out
    check(st, f"mhc_debug_bounds {out}")
    return out


def read_device_status(ws: torch.Tensor, stream: torch.cuda.Stream) -> int:
    out = ctypes.c_int(0)
    check(load().mhc_read_device_status(ws.data_ptr(), stream.cuda_stream, ctypes.byref(out)),
          "mhc_read_device_status")
    return int(out.value)
