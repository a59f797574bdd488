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


def _bwd_grid(T, D, sms=SMS):
    g = (ctypes.c_int32 * 6)()
    assert _lib.load().mhc_query_bwd_grid(T, 4, D, sms, g) == 0
    return tuple(g)


def _bwd_units(T, D, sms=SMS):
    """The (tile, d-slice) units of every CTA of the n = 4 tensor-core
    backward, with the G-partial slot each CTA writes, as the kernel walks them."""
    Dc, S_K, S_T, J, E, R = _bwd_grid(T, D, sms)
    tiles = max(1, -(-T // 128))
    ctas = []
    for b in range(S_K * S_T + E):
        if b >= S_K * S_T:
            e = b - S_K * S_T
            units = [(R - 1 - u % R, e * (S_K // E) + u // R) for u in range(S_K // E * R)]
            slot = S_T
        else:
            s, g = b % S_K, b // S_K
            count = J if E else ((tiles - 1 - g) // S_T + 1 if g < tiles else 0)
            units = [(tiles - 1 - (g + u * S_T), s) for u in range(count)]
            slot = g
        ctas.append((slot, units))
    return (Dc, S_K, S_T, J, E, R), tiles, ctas


@pytest.mark.parametrize("T", [1, 128, 1350, 1408, 4096, 5888, 16384, 32768, 100000])
@pytest.mark.parametrize("D", [1024, 4096, 7168])
@pytest.mark.parametrize("sms", [74, 144, 148])
def test_bwd_grid_covers_every_unit_once_and_balances(T, D, sms):
    """Every (tile, d-slice) unit is done by exactly one CTA, every (slot,
    d-slice) G partial has exactly one writer, the grid fits one wave, and no
    CTA does more units than round robin over the token groups would give."""
    (Dc, S_K, S_T, J, E, R), tiles, ctas = _bwd_units(T, D, sms)
    assert D == S_K * Dc and len(ctas) <= max(sms, S_K)
    seen, writers = {}, {}
    for b, (slot, units) in enumerate(ctas):
        for t, s in units:
            assert 0 <= t < tiles and 0 <= s < S_K
            assert (t, s) not in seen, (t, s)
            seen[(t, s)] = b
            writers.setdefault((slot, s), set()).add(b)
    assert len(seen) == tiles * S_K
    assert all(len(w) == 1 for w in writers.values())
    busiest = max(len(u) for _, u in ctas)
    assert busiest <= -(-tiles // S_T) * -(-(S_K * S_T) // sms)
    if E:
        assert busiest < -(-tiles // S_T)     # the leftover CTAs are only taken when they help


def test_bwd_grid_at_the_llm_shape_fills_the_sms():
    (Dc, S_K, S_T, J, E, R), tiles, ctas = _bwd_units(16384, 4096)
    assert len(ctas) == SMS and E > 0 and R > 0
    assert max(len(u) for _, u in ctas) == -(-tiles * S_K // SMS)   # 14 = ceil(2048 / 148): no CTA above the ideal
    assert plan(1, 16384, 4, 4096)["ctas"] == SMS


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
