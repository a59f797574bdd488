"""Parity of the CUDA path (through the C ABI) with the reference golden / CPU oracle.

* every golden fixture (outputs of the reference's own golden, tests/golden/);
* the reference's README backward shapes and larger shapes against the oracle
  run live on the same seeded inputs;
* at the full LLM size, size-independent properties: per-token outputs of a
  random token sample against the oracle, shard additivity of the parameter
  gradients, bitwise determinism.
* the wide configuration (n=8, D=4096, B=2, S=8192) and the 8-GPU row width
  (n=4, D=7168, 4096 tokens) over every token, in shards against the oracle.
Tolerances: fp32 outputs max|a-b|/max|ref| <= 1e-4; bf16 h_in/dx within 1 bf16
ulp of the golden value, or, for at most 0.1% of the elements (cancellation),
within the fp32 accumulation floor 2^-18 * sum|terms|; the counts are printed
at the end of the run.
"""
import numpy as np
import pytest
import torch

from mhc_ops_b200 import _lib, mhc_backward_manual, mhc_forward_pre
from mhc_ops_b200.synthetic import make_inputs
from oracle import mhc_oracle as O
from tests._golden import fixture_names, load_fixture
from tests._gpu import (BF16_REPORT, DEV, FLOOR_FRAC, FP32_TOL, assert_bwd_close, assert_fwd_close, bits, check_bf16,
                        from_bits, oracle_shards, rel)

pytestmark = pytest.mark.gpu


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _run_fwd_bwd_on_fixture(z):
    x = from_bits(z["x"])
    out = mhc_forward_pre(x, _t(z["phi"]), _t(z["alpha"]), _t(z["bias"]), outflag=True)
    bout = mhc_backward_manual(x, _t(z["phi"]), _t(z["alpha"]), _t(z["bias"]), _t(z["inv_rms"]),
                               _t(z["h_mix"]), _t(z["h_pre"]), _t(z["h_post"]), from_bits(z["dh_in"]),
                               _t(z["dh_post"]), _t(z["dh_res"]), _t(z["gamma"]))
    torch.cuda.synchronize()
    return out, bout


@pytest.mark.parametrize("name", fixture_names())
def test_fixture_parity_with_reference_golden(name):
    z = load_fixture(name)
    out, bout = _run_fwd_bwd_on_fixture(z)
    ref = (z["h_in"], z["h_post"], z["h_res"], z["inv_rms"], z["h_mix"], z["h_pre"])
    assert_fwd_close(out, ref, z["x"], tag=name)
    scale = O.backward_term_scale(z["x"], z["phi"], z["alpha"], z["inv_rms"], z["h_mix"], z["h_pre"],
                                  z["h_post"], z["dh_in"], z["dh_post"], z["dh_res"], z["gamma"])
    assert_bwd_close(bout, (z["dx"], z["dphi"], z["dalpha"], z["dbias"], z["dgamma"]), scale, tag=name)


def _live_case(B, S, n, D, seed, gamma=True):
    inp = make_inputs(B, S, n, D, seed=seed)
    xb = bits(inp.x)
    ref_f = O.forward(xb, inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), outflag=True)
    g = inp.gamma.to(DEV) if gamma else None
    gnp = inp.gamma.numpy() if gamma else np.ones((n, D), np.float32)
    d = inp.to(DEV)
    out = mhc_forward_pre(d.x, d.phi, d.alpha, d.bias, outflag=True)
    # backward from the oracle's forward intermediates, so the two halves are checked separately
    inv_rms, h_mix, h_pre, h_post = (_t(ref_f[3]), _t(ref_f[4]), _t(ref_f[5]), _t(ref_f[1]))
    bout = mhc_backward_manual(d.x, d.phi, d.alpha, d.bias, inv_rms, h_mix, h_pre, h_post, d.dh_in, d.dh_post,
                               d.dh_res, g)
    torch.cuda.synchronize()
    ref_b = O.backward(xb, inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), ref_f[3], ref_f[4], ref_f[5],
                       ref_f[1], bits(inp.dh_in), inp.dh_post.numpy(), inp.dh_res.numpy(), gnp)
    scale = O.backward_term_scale(xb, inp.phi.numpy(), inp.alpha.numpy(), ref_f[3], ref_f[4], ref_f[5], ref_f[1],
                                  bits(inp.dh_in), inp.dh_post.numpy(), inp.dh_res.numpy(), gnp)
    tag = f"{B}x{S}x{n}x{D}"
    assert_fwd_close(out, ref_f, xb, tag=tag)
    assert_bwd_close(bout, ref_b, scale, tag=tag)


@pytest.mark.parametrize("B,S,D", [(2, 64, 128), (2, 256, 256), (1, 1024, 512), (1, 2048, 512)])
def test_readme_backward_shapes_vs_oracle(B, S, D):
    _live_case(B, S, 4, D, seed=11)


@pytest.mark.parametrize("B,S,n,D,gamma", [
    (1, 384, 4, 4096, True),     # LLM row width, a slice of the token count
    (1, 160, 4, 7168, True),     # 8-GPU config row width
    (1, 160, 8, 4096, True),     # wider hyper-connection n=8 (N=80)
    (1, 130, 4, 1024, False),    # gamma=None, token count not a multiple of 128
    (3, 1, 4, 64, True),         # a handful of tokens
    (1, 33, 2, 40, True),        # n=2, D not a multiple of 64
    (1, 50, 3, 24, True),        # odd n
    (1, 300, 8, 1024, False),    # n=8 tiled backward, ragged token tiles, gamma=None
    (1, 70, 6, 512, True),       # n=6 tiled backward
    (1, 200, 5, 256, True),      # odd n on the tensor cores: dx one 64-k block at a time
    (1, 140, 2, 128, False),     # n=2: dx in stream pairs, one pair per d-block
    (1, 200, 4, 9536, True),     # n=4, a row wider than the 8-GPU config's (149 64-wide d-blocks per stream)
])
def test_wide_rows_vs_oracle(B, S, n, D, gamma):
    _live_case(B, S, n, D, seed=12, gamma=gamma)


@pytest.mark.parametrize("B,S,n,D", [(1, 64, 1, 64), (1, 200, 2, 256), (2, 75, 3, 512), (1, 130, 5, 256),
                                     (1, 100, 6, 128), (1, 70, 7, 192)])
def test_every_stream_count_on_the_tensor_core_forward_vs_oracle(B, S, n, D):
    """n outside {4, 8} with D a multiple of 64: the projection on the tensor
    cores and the row kernel (the generic kernels only for other D), ragged
    token tiles; forward and backward against the oracle."""
    assert _lib.query_plan(0, B * S, n, D)["path"] == "tensor-core"
    _live_case(B, S, n, D, seed=17)


@pytest.mark.parametrize("B,S,D", [(1, 1350, 4096), (1, 1664, 2048), (1, 5888, 1024)])
def test_backward_with_leftover_tile_ctas_vs_oracle(B, S, D):
    """Token counts whose 128-token tiles do not split evenly over the token
    groups of the n = 4 tensor-core backward: the leftover tiles run on extra
    CTAs (whole d-slices each, their own slot of the G partials); forward and
    backward against the oracle over all tokens (1350: a ragged last tile)."""
    q = _lib.query_plan(1, B * S, 4, D)
    assert q["path"] == "tensor-core" and q["leftover_ctas"] > 0, q
    _live_case(B, S, 4, D, seed=19)


@pytest.mark.parametrize("B,S,n,D", [(1, 4096, 4, 2560), (2, 2048, 8, 1280)])
def test_reference_forward_test_shapes_vs_oracle(B, S, n, D):
    """The largest shapes of the reference's forward tests
    (test/forward/test_forward.py:460-483), forward and backward, all tokens."""
    _live_case(B, S, n, D, seed=13)


def test_full_llm_size_properties():
    """B=4,S=4096,n=4,D=4096: sampled tokens vs oracle, shard additivity, determinism."""
    B, S, n, D = 4, 4096, 4, 4096
    inp = make_inputs(B, S, n, D, seed=0)
    d = inp.to(DEV)
    out = mhc_forward_pre(d.x, d.phi, d.alpha, d.bias, outflag=True)
    bw = mhc_backward_manual(d.x, d.phi, d.alpha, d.bias, out[3], out[4], out[5], out[1], d.dh_in, d.dh_post,
                             d.dh_res, d.gamma)
    bw2 = mhc_backward_manual(d.x, d.phi, d.alpha, d.bias, out[3], out[4], out[5], out[1], d.dh_in,
                              d.dh_post, d.dh_res, d.gamma)
    torch.cuda.synchronize()
    for a, b in zip(bw, bw2):
        assert torch.equal(a, b), "backward is not bitwise deterministic"

    # per-token outputs of a token sample against the oracle
    T = B * S
    rng = np.random.default_rng(0)
    idx = np.sort(rng.choice(T, size=96, replace=False))
    xs = inp.x.reshape(T, n, D)[idx].unsqueeze(0)
    ref_f = O.forward(bits(xs), inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), outflag=True)
    sel = [o.reshape(T, *o.shape[2:])[torch.as_tensor(idx, device=DEV)].unsqueeze(0) for o in out]
    assert_fwd_close(sel, ref_f, bits(xs), tag="llm-sample")
    ref_b = O.backward(bits(xs), inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), ref_f[3], ref_f[4],
                       ref_f[5], ref_f[1], bits(inp.dh_in.reshape(T, D)[idx].unsqueeze(0)),
                       inp.dh_post.reshape(T, n)[idx][None].numpy(), inp.dh_res.reshape(T, n, n)[idx][None].numpy(),
                       inp.gamma.numpy())
    scale = O.backward_term_scale(bits(xs), inp.phi.numpy(), inp.alpha.numpy(), ref_f[3], ref_f[4], ref_f[5],
                                  ref_f[1], bits(inp.dh_in.reshape(T, D)[idx].unsqueeze(0)),
                                  inp.dh_post.reshape(T, n)[idx][None].numpy(),
                                  inp.dh_res.reshape(T, n, n)[idx][None].numpy(), inp.gamma.numpy())
    dx_s = bw[0].reshape(T, n, D)[torch.as_tensor(idx, device=DEV)]
    check_bf16("llm-sample", "dx", bits(dx_s), ref_b[0].reshape(-1, n, D), scale.reshape(-1, n, D))

    # parameter gradients are sums over tokens: 4 shards must add up to the whole
    parts = []
    for k in range(4):
        sl = slice(k * S, (k + 1) * S)
        f = lambda t: t.reshape(T, *t.shape[2:])[sl].unsqueeze(0)  # noqa: E731
        parts.append(mhc_backward_manual(f(d.x), d.phi, d.alpha, d.bias, f(out[3].unsqueeze(-1)).squeeze(-1),
                                         f(out[4]), f(out[5]), f(out[1]), f(d.dh_in), f(d.dh_post), f(d.dh_res),
                                         d.gamma))
    torch.cuda.synchronize()
    for j in range(1, 5):
        summed = sum(p[j].double() for p in parts)
        assert rel(bw[j], summed.cpu().numpy()) <= FP32_TOL, j
    # dgamma / dphi of the first shard against the oracle (512 tokens)
    sl = slice(0, 512)
    f = lambda t: t.reshape(T, *t.shape[2:])[sl].unsqueeze(0)  # noqa: E731
    xs = f(inp.x)
    rf = O.forward(bits(xs), inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), outflag=True)
    rb = O.backward(bits(xs), inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), rf[3], rf[4], rf[5], rf[1],
                    bits(f(inp.dh_in)), f(inp.dh_post).numpy(), f(inp.dh_res).numpy(), inp.gamma.numpy())
    ob = mhc_backward_manual(f(d.x), d.phi, d.alpha, d.bias, _t(rf[3]), _t(rf[4]), _t(rf[5]), _t(rf[1]),
                             f(d.dh_in), f(d.dh_post), f(d.dh_res), d.gamma)
    torch.cuda.synchronize()
    for j in range(1, 5):
        assert rel(ob[j], rb[j]) <= FP32_TOL, j


def test_zero_tokens():
    inp = make_inputs(1, 0, 4, 64, seed=1).to(DEV)
    out = mhc_forward_pre(inp.x, inp.phi, inp.alpha, inp.bias, outflag=True)
    assert out[0].shape == (1, 0, 64)
    bw = mhc_backward_manual(inp.x, inp.phi, inp.alpha, inp.bias, out[3], out[4], out[5], out[1], inp.dh_in,
                             inp.dh_post, inp.dh_res, inp.gamma)
    torch.cuda.synchronize()
    assert bw[0].shape == (1, 0, 4, 64)
    for g in bw[1:]:
        assert torch.count_nonzero(g) == 0


def test_outflag_false_returns_three():
    inp = make_inputs(1, 5, 4, 64, seed=2).to(DEV)
    out = mhc_forward_pre(inp.x, inp.phi, inp.alpha, inp.bias)
    assert len(out) == 3
    full = mhc_forward_pre(inp.x, inp.phi, inp.alpha, inp.bias, outflag=True)
    for a, b in zip(out, full[:3]):
        assert torch.equal(a, b)


def _full_batch_vs_oracle(B, S, n, D, seed, shard, tag):
    """Forward and backward of the whole batch on the GPU; every token checked
    against the oracle, shard by shard in worker processes (the oracle's
    backward runs from the GPU's forward intermediates, so both backward
    implementations see the same inputs); parameter gradients against the
    float64 sum of the oracle's per-shard gradients."""
    inp = make_inputs(B, S, n, D, seed=seed)
    d = inp.to(DEV)
    out = mhc_forward_pre(d.x, d.phi, d.alpha, d.bias, outflag=True)
    bw = mhc_backward_manual(d.x, d.phi, d.alpha, d.bias, out[3], out[4], out[5], out[1], d.dh_in, d.dh_post,
                             d.dh_res, d.gamma)
    torch.cuda.synchronize()
    T = B * S
    N = n * n + 2 * n
    phi, alpha, bias, gamma = inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), inp.gamma.numpy()
    xb = bits(inp.x).reshape(T, n, D)
    dhb = bits(inp.dh_in).reshape(T, D)
    dpost = inp.dh_post.reshape(T, n).numpy()
    dres = inp.dh_res.reshape(T, n, n).numpy()
    h_in_b = bits(out[0]).reshape(T, D)
    f_np = [o.reshape(T, *o.shape[2:]).cpu().numpy() for o in out[1:]]
    dx_b = bits(bw[0]).reshape(T, n, D)
    jobs, bounds = [], []
    for a in range(0, T, shard):
        sl = slice(a, min(T, a + shard))
        bounds.append((a, sl.stop))
        jobs.append((xb[sl][None], dhb[sl][None], dpost[sl][None], dres[sl][None], phi, alpha, bias, gamma,
                     h_in_b[sl][None], tuple(o[sl][None] for o in f_np), dx_b[sl][None]))
    sums = [np.zeros((N, n * D)), np.zeros(3), np.zeros(N), np.zeros(n * D)]
    for (a, b), res in zip(bounds, oracle_shards(jobs)):
        for nm, e in res["fwd_rel"].items():
            assert e <= FP32_TOL, f"{tag} [{a}:{b}] {nm}: rel err {e:.3g}"
        for nm in ("h_in", "dx"):
            st = res[nm]
            BF16_REPORT.append((f"{tag} [{a}:{b}]", nm, st))
            assert st["bad"] == 0, f"{tag} [{a}:{b}] {nm}: {st['bad']} beyond tolerance ({st})"
            assert st["floor_needed"] <= FLOOR_FRAC * st["n"] + 8, f"{tag} [{a}:{b}] {nm}: {st}"
        for acc, r in zip(sums, res["param"]):
            acc += r.reshape(acc.shape)
    for name, o, r in zip(("dphi", "dalpha", "dbias", "dgamma"), bw[1:], sums):
        e = rel(o, r)
        assert e <= FP32_TOL, f"{tag} {name}: rel err {e:.3g}"


def test_wide_config_full_size_vs_oracle():
    """The wide configuration, n=8, D=4096, B=2, S=8192 (16384 tokens, N=80):
    every token's forward outputs and dx against the oracle, and the parameter
    gradients of the whole batch (the tiled backward with its multi-group
    parameter-gradient partials)."""
    _full_batch_vs_oracle(2, 8192, 8, 4096, seed=21, shard=1024, tag="wide n8 D4096")


def test_eight_gpu_row_width_vs_oracle():
    """The 8-GPU configuration's row width, n=4, D=7168, over 4096 tokens
    (one GPU's share of B=8,S=4096 at 8 GPUs): every token against the oracle."""
    _full_batch_vs_oracle(1, 4096, 4, 7168, seed=22, shard=1024, tag="8gpu n4 D7168")


@pytest.mark.parametrize("B,S,n,D", [(4, 4096, 4, 4096), (1, 300, 8, 1024), (1, 50, 3, 24), (1, 130, 4, 1024)])
def test_backward_recomputing_intermediates_equals_stored_form(B, S, n, D):
    """mhc_backward_manual with inv_rms, h_mix, h_pre (and h_post) None runs the
    forward kernels first: the gradients must equal, bit for bit, those of the
    backward given the intermediates mhc_forward_pre(outflag=True) stored
    (src/forward/golden.py:65-69 is the stored contract); and, on a token
    sample, the oracle."""
    inp = make_inputs(B, S, n, D, seed=31)
    d = inp.to(DEV)
    out = mhc_forward_pre(d.x, d.phi, d.alpha, d.bias, outflag=True)
    stored = mhc_backward_manual(d.x, d.phi, d.alpha, d.bias, out[3], out[4], out[5], out[1], d.dh_in, d.dh_post,
                                 d.dh_res, d.gamma)
    recomputed = mhc_backward_manual(d.x, d.phi, d.alpha, d.bias, None, None, None, None, d.dh_in, d.dh_post,
                                     d.dh_res, d.gamma)
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(stored, recomputed)):
        assert torch.equal(a, b), f"output {i} of the recomputing backward differs"
    if B * S <= 2048:
        ref_f = O.forward(bits(inp.x), inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), outflag=True)
        ref_b = O.backward(bits(inp.x), inp.phi.numpy(), inp.alpha.numpy(), inp.bias.numpy(), ref_f[3], ref_f[4],
                           ref_f[5], ref_f[1], bits(inp.dh_in), inp.dh_post.numpy(), inp.dh_res.numpy(),
                           inp.gamma.numpy())
        scale = O.backward_term_scale(bits(inp.x), inp.phi.numpy(), inp.alpha.numpy(), ref_f[3], ref_f[4], ref_f[5],
                                      ref_f[1], bits(inp.dh_in), inp.dh_post.numpy(), inp.dh_res.numpy(),
                                      inp.gamma.numpy())
        assert_bwd_close(recomputed, ref_b, scale, tag=f"recompute {B}x{S}x{n}x{D}")
