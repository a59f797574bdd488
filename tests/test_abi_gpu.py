"""The C ABI called directly with raw device pointers (as a cgo/ctypes user would),
and its error paths on a GPU."""
import ctypes

import pytest
import torch

from mhc_ops_b200 import _lib, mhc_forward_pre
from mhc_ops_b200.synthetic import make_inputs

pytestmark = pytest.mark.gpu


def _fwd_args(d, outs, ws, T, n, D):
    return _lib.FwdArgs(x=d.x.data_ptr(), phi=d.phi.data_ptr(), alpha=d.alpha.data_ptr(),
                        bias=d.bias.data_ptr(), h_in=outs[0].data_ptr(), h_post=outs[1].data_ptr(),
                        h_res=outs[2].data_ptr(), inv_rms=None, h_mix=None, h_pre=None, tokens=T, n=n, D=D,
                        norm_eps=1e-6, hc_eps=1e-6, workspace=ws.data_ptr(), workspace_bytes=ws.numel())


def test_raw_abi_forward_matches_python_api():
    lib = _lib.load()
    B, S, n, D = 1, 40, 4, 512
    d = make_inputs(B, S, n, D, seed=3).to("cuda")
    T = B * S
    outs = (torch.empty(T, D, dtype=torch.bfloat16, device="cuda"), torch.empty(T, n, device="cuda"),
            torch.empty(T, n, n, device="cuda"))
    size = ctypes.c_size_t(0)
    assert lib.mhc_fwd_workspace_size(T, n, D, ctypes.byref(size)) == 0
    ws = torch.zeros(size.value, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.mhc_fwd(ctypes.byref(_fwd_args(d, outs, ws, T, n, D)), stream) == 0
    ref = mhc_forward_pre(d.x, d.phi, d.alpha, d.bias)
    torch.cuda.synchronize()
    assert torch.equal(outs[0].view(1, S, D), ref[0])
    assert torch.equal(outs[1].view(1, S, n), ref[1])
    status = ctypes.c_int(-1)
    assert lib.mhc_read_device_status(ws.data_ptr(), stream, ctypes.byref(status)) == 0
    assert status.value == 0


def test_abi_rejects_bad_arguments():
    lib = _lib.load()
    B, S, n, D = 1, 8, 4, 64
    d = make_inputs(B, S, n, D, seed=4).to("cuda")
    T = B * S
    outs = (torch.empty(T, D, dtype=torch.bfloat16, device="cuda"), torch.empty(T, n, device="cuda"),
            torch.empty(T, n, n, device="cuda"))
    size = ctypes.c_size_t(0)
    lib.mhc_fwd_workspace_size(T, n, D, ctypes.byref(size))
    ws = torch.zeros(size.value, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    a = _fwd_args(d, outs, ws, T, n, D)
    a.workspace_bytes = 16
    assert lib.mhc_fwd(ctypes.byref(a), stream) == 4            # workspace too small
    a = _fwd_args(d, outs, ws, T, n, D)
    a.n = 9
    assert lib.mhc_fwd(ctypes.byref(a), stream) == 2            # bad shape
    a = _fwd_args(d, outs, ws, T, n, D)
    a.phi = d.phi.data_ptr() + 1
    assert lib.mhc_fwd(ctypes.byref(a), stream) == 3            # misaligned
    a = _fwd_args(d, outs, ws, T, n, D)
    a.x = None
    assert lib.mhc_fwd(ctypes.byref(a), stream) == 1            # NULL input
    with pytest.raises(ValueError):
        mhc_forward_pre(d.x, d.phi[:, :-1].contiguous(), d.alpha, d.bias)   # wrong phi shape


@pytest.mark.parametrize("which,T,n,D,path", [
    (0, 16384, 4, 4096, "tensor-core-fused"),   # the LLM config: one cooperative launch
    (0, 16384, 8, 4096, "tensor-core"),         # n = 8: projection + row kernel
    (0, 1000, 6, 512, "tensor-core"),          # every n: projection + row kernel
    (0, 1000, 6, 100, "generic"),              # D not a multiple of 64
    (1, 16384, 4, 4096, "tensor-core"),
    (1, 16384, 8, 4096, "tiled"),               # n = 8 backward: the n != 4 tcgen05 kernels
    (1, 100, 4, 36, "generic"),                 # D not a multiple of 8
])
def test_launch_plan_routes_each_shape(which, T, n, D, path):
    """The plan query names the kernels a shape runs on (no kernel is launched),
    and the device-free query at this device's SM count gives the same plan."""
    got = _lib.query_plan(which, T, n, D)
    assert got["path"] == path
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert _lib.query_plan(which, T, n, D, sms=sms) == got


def test_launch_counter_advances():
    d = make_inputs(1, 16, 4, 128, seed=5).to("cuda")
    before = _lib.launch_count()
    mhc_forward_pre(d.x, d.phi, d.alpha, d.bias)
    torch.cuda.synchronize()
    assert _lib.launch_count() > before


def test_bounded_wait_expiry_reports_timeout():
    """A device wait that can never complete gives up (about a second), records
    MHC_ERR_DEVICE_TIMEOUT in the workspace status word, and leaves the context
    usable: the next forward call still works and the status word was cleared."""
    lib = _lib.load()
    stream = torch.cuda.current_stream()
    ws = torch.zeros(1 << 12, dtype=torch.uint8, device="cuda")
    assert lib.mhc_selftest_wait_expiry(ws.data_ptr(), stream.cuda_stream) == 0
    torch.cuda.synchronize()
    assert int(ws[4:8].view(torch.int32).item()) == 3, "both bounded waits (mbarrier, counter) must report"
    assert _lib.read_device_status(ws, stream) == _lib.MHC_ERR_DEVICE_TIMEOUT
    assert _lib.read_device_status(ws, stream) == 0          # read clears it
    d = make_inputs(1, 16, 4, 128, seed=6).to("cuda")
    out = mhc_forward_pre(d.x, d.phi, d.alpha, d.bias)
    torch.cuda.synchronize()
    assert torch.isfinite(out[1]).all()


def test_timeout_reported_through_the_python_api():
    """The Python API surfaces a device timeout: the status word of the cached
    workspace is set (by the bounded-wait self test, which gives up after
    about a second, no fault), the next forward through mhc_forward_pre copies
    it, and check_device_status raises MHC_ERR_DEVICE_TIMEOUT.  The word is
    cleared by the raise, so the calls after it run clean."""
    lib = _lib.load()
    stream = torch.cuda.current_stream()
    d = make_inputs(1, 16, 4, 128, seed=7).to("cuda")
    mhc_forward_pre(d.x, d.phi, d.alpha, d.bias)
    _lib.check_device_status()
    ws = _lib._ws_cache[(torch.cuda.current_device(), stream.cuda_stream)]
    assert lib.mhc_selftest_wait_expiry(ws.buf.data_ptr(), stream.cuda_stream) == 0
    mhc_forward_pre(d.x, d.phi, d.alpha, d.bias)
    with pytest.raises(_lib.MhcError) as err:
        _lib.check_device_status()
    assert err.value.status == _lib.MHC_ERR_DEVICE_TIMEOUT
    out = mhc_forward_pre(d.x, d.phi, d.alpha, d.bias)
    _lib.check_device_status()
    assert torch.isfinite(out[1]).all()
