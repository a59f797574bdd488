"""Launch-plan host logic, on the CPU: which kernels each shape runs on and the
cost models behind the grids, from the device-free plan query at B200's 148
SMs (mhc_query_plan_for; the GPU test checks it against mhc_query_plan)."""
import ctypes

import pytest

from mhc_ops_b200 import _lib

SMS = 148   # B200


def plan(which, T, n, D, sms=SMS):
    return _lib.query_plan(which, T, n, D, sms=sms)


def test_llm_shape_runs_the_fused_forward_and_the_tensor_core_backward():
    f = plan(0, 16384, 4, 4096)
    assert f["path"] == "tensor-core-fused" and f["ctas"] == SMS
    assert (4 * 4096 // 64) % f["k_slices"] == 0   # K-slices split the 64-wide K blocks evenly
    b = plan(1, 16384, 4, 4096)
    assert b["path"] == "tensor-core"
    # d-slices x token groups fill the SMs without a second wave
    assert b["d_slices"] * b["token_groups"] <= SMS
    assert 4096 % b["d_slices"] == 0 and (4096 // b["d_slices"]) % 64 == 0


def test_wide_and_other_shapes_route_as_documented():
    assert plan(0, 16384, 8, 4096)["path"] == "tensor-core"        # n = 8: projection + row kernel
    b = plan(1, 16384, 8, 4096)
    assert b["path"] == "tiled" and 1 <= b["token_groups"] <= 8
    assert b["dx"] == "tensor-core-stream-pairs"                   # even n: dx in stream pairs
    assert plan(1, 200, 5, 256)["dx"] == "tensor-core"              # odd n: one 64-k block at a time
    assert plan(1, 33, 2, 40)["dx"] == "cuda-cores"                 # D not a multiple of 64
    assert plan(1, 70, 6, 512)["path"] == "tiled"
    for n in (1, 2, 3, 5, 6, 7):                                    # every n: projection + row kernel
        assert plan(0, 1000, n, 512)["path"] == "tensor-core"
    assert plan(0, 1000, 6, 100)["path"] == "generic"              # D not a multiple of 64
    assert plan(1, 100, 4, 36)["path"] == "generic"                # D not a multiple of 8
    assert plan(1, 100, 4, 40)["path"] == "tiled"                  # n = 4, D % 64 != 0: the n != 4 kernels
    assert plan(0, 16384, 4, 7168)["path"] == "tensor-core-fused"  # the 8-GPU row width


@pytest.mark.parametrize("T", [1, 127, 128, 4096, 16384, 100000])
def test_plans_scale_with_tokens_and_sms(T):
    for sms in (1, 74, 148):
        f = plan(0, T, 4, 4096, sms=sms)
        assert 1 <= f["ctas"] <= sms
        b = plan(1, T, 4, 4096, sms=sms)
        assert b["d_slices"] * b["token_groups"] <= max(sms, b["d_slices"])


def test_bwd_workspace_grows_with_tokens():
    lib = _lib.load()
    sizes = []
    for T in (128, 4096, 16384):
        out = ctypes.c_size_t(0)
        assert lib.mhc_bwd_workspace_size_for(T, 4, 4096, SMS, ctypes.byref(out)) == 0
        sizes.append(out.value)
    assert sizes[0] < sizes[1] < sizes[2]
    out = ctypes.c_size_t(0)
    assert lib.mhc_bwd_workspace_size_for(16384, 8, 4096, SMS, ctypes.byref(out)) == 0 and out.value > 0


def test_plan_query_rejects_bad_arguments():
    lib = _lib.load()
    p, c, k = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    assert lib.mhc_query_plan_for(2, 128, 4, 64, SMS, ctypes.byref(p), ctypes.byref(c), ctypes.byref(k)) == 2
    assert lib.mhc_query_plan_for(0, 128, 9, 64, SMS, ctypes.byref(p), ctypes.byref(c), ctypes.byref(k)) == 2
    assert lib.mhc_query_plan_for(0, 128, 4, 64, 0, ctypes.byref(p), ctypes.byref(c), ctypes.byref(k)) == 2
    assert lib.mhc_query_plan_for(0, 128, 4, 64, SMS, None, ctypes.byref(c), ctypes.byref(k)) == 1
