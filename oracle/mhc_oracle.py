"""CPU oracle for the mHC pre-op (forward and backward).  TEST INFRASTRUCTURE ONLY.

This module is the checker.  It is imported only by ``tests/``, by
``__graft_entry__.smoke()`` and by the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py``.  The product path (``mhc_ops_b200``) never imports it and
has no CPU fallback.

It restates, in numpy float32, the reference golden path of folrent1896/mhc_ops:

* forward  : ``src/forward/golden.py:34-69``  (``mhc_forward_pre``)
* backward : ``src/backward/golden.py:38-96`` (``mhc_backward_manual``)

keeping the golden's operation order (pre-RMS projection, ``sigmoid + hc_eps``,
``2 * sigmoid``, ``h_post * (1 - h_post / 2)``, the flat ``[nD]`` dgamma and
the final bf16 casts).  bf16 tensors are carried as ``uint16`` bit patterns;
``bf16_to_f32`` widens exactly and ``f32_to_bf16`` rounds to nearest-even, as
``torch.Tensor.to(torch.bfloat16)`` does.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference golden
(PyTorch, CPU) on seeded inputs and stores inputs and outputs as fixtures;
``tests/test_oracle_golden.py`` checks this oracle against every fixture.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "bf16_to_f32",
    "f32_to_bf16",
    "n_out",
    "forward",
    "backward",
    "bf16_stats",
    "bf16_within",
]


# --------------------------------------------------------------------------- bf16
def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    """Exact widening of bf16 bit patterns (uint16) to float32."""
    u16 = np.ascontiguousarray(u16, dtype=np.uint16)
    return (u16.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16(f32: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (round-to-nearest-even); returns uint16 bit patterns."""
    f32 = np.ascontiguousarray(f32, dtype=np.float32)
    u = f32.view(np.uint32)
    nan = np.isnan(f32)
    rounded = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    if nan.any():
        rounded = np.where(nan, ((u >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16), rounded)
    return rounded


def n_out(n: int) -> int:
    """Width of the projection, n^2 + 2n (golden.py:17 ``phi: [n^2 + 2n, nD]``)."""
    return n * n + 2 * n


def _sigmoid(v: np.ndarray) -> np.ndarray:
    one = np.float32(1.0)
    return one / (one + np.exp(-v, dtype=np.float32))


# ------------------------------------------------------------------------ forward
def forward(x_bf16, phi, alpha, bias, outflag=False, norm_eps=1e-6, hc_eps=1e-6):
    """Restatement of ``src/forward/golden.py:10-69``.

    x_bf16: uint16 [B,S,n,D]; phi float32 [N,nD]; alpha float32 [3]; bias float32 [N].
    Returns (h_in u16 [B,S,D], h_post [B,S,n], h_res [B,S,n,n]) and, when
    ``outflag``, additionally (inv_rms [B,S], h_mix [B,S,N], h_pre [B,S,n]).
    """
    B, S, n, D = x_bf16.shape
    nD = n * D
    phi = np.asarray(phi, dtype=np.float32)
    alpha = np.asarray(alpha, dtype=np.float32)
    bias = np.asarray(bias, dtype=np.float32)
    f32 = np.float32

    x_f = bf16_to_f32(x_bf16)                                   # x.float()
    vecX = x_f.reshape(B, S, nD)                                # golden.py:38
    h_mix = np.matmul(vecX, phi.T)                              # golden.py:41 (pre-RMS)
    ms = np.mean(np.square(vecX), axis=-1, keepdims=True, dtype=np.float32)
    inv_rms = (f32(1.0) / np.sqrt(ms + f32(norm_eps))).astype(np.float32)   # golden.py:44
    h_mix_tmp = h_mix * inv_rms                                 # golden.py:45

    h_pre1 = h_mix_tmp[..., :n]                                 # golden.py:48
    h_post1 = h_mix_tmp[..., n:2 * n]
    h_res1 = h_mix_tmp[..., 2 * n:]
    h_res2 = h_res1.reshape(B, S, n, n)                         # golden.py:49
    a_pre, a_post, a_res = alpha[0], alpha[1], alpha[2]         # golden.py:50

    h_pre2 = a_pre * h_pre1 + bias[:n]                          # golden.py:53
    h_post2 = a_post * h_post1 + bias[n:2 * n]                  # golden.py:54
    h_res = a_res * h_res2 + bias[2 * n:].reshape(n, n)         # golden.py:55

    h_pre = _sigmoid(h_pre2) + f32(hc_eps)                      # golden.py:58
    h_post = f32(2.0) * _sigmoid(h_post2)                       # golden.py:59

    h_in_fp = (h_pre[..., None] * x_f).sum(axis=2, dtype=np.float32)   # golden.py:62
    h_in = f32_to_bf16(h_in_fp)                                 # golden.py:63

    h_post = h_post.astype(np.float32)
    h_res = h_res.astype(np.float32)
    if not outflag:
        return h_in, h_post, h_res
    return (h_in, h_post, h_res, inv_rms[..., 0].astype(np.float32),
            h_mix.astype(np.float32), h_pre.astype(np.float32))   # golden.py:65-69


# ----------------------------------------------------------------------- backward
def backward(x_bf16, phi, alpha, bias, inv_rms, h_mix, h_pre, h_post,
             dh_in_bf16, dh_post, dh_res, gamma, norm_eps=1e-6, hc_eps=1e-6):
    """Restatement of ``src/backward/golden.py:10-96``.

    Returns (dx u16 [B,S,n,D], dphi [N,nD], dalpha [3], dbias [N], dgamma [nD]).
    ``dgamma`` is flat ``[n*D]`` exactly as the golden returns it (golden.py:93).
    ``bias`` and ``norm_eps`` are accepted for signature parity; the golden
    does not use them either.
    """
    del bias, norm_eps
    B, S, n, D = x_bf16.shape
    nD = n * D
    T = B * S
    f32 = np.float32
    phi = np.asarray(phi, dtype=np.float32)
    alpha = np.asarray(alpha, dtype=np.float32)
    inv_rms = np.asarray(inv_rms, dtype=np.float32)
    h_mix = np.asarray(h_mix, dtype=np.float32)
    h_pre = np.asarray(h_pre, dtype=np.float32)
    h_post = np.asarray(h_post, dtype=np.float32)
    dh_post = np.asarray(dh_post, dtype=np.float32)
    dh_res = np.asarray(dh_res, dtype=np.float32)
    gamma = np.asarray(gamma, dtype=np.float32)

    x_fp = bf16_to_f32(x_bf16)                                  # golden.py:49
    vecX = x_fp.reshape(B, S, nD)                               # golden.py:40
    a_pre, a_post, a_res = alpha[0], alpha[1], alpha[2]         # golden.py:41

    h_in_fp_grad = bf16_to_f32(dh_in_bf16)                      # golden.py:50
    dh_pre = (h_in_fp_grad[:, :, None, :] * x_fp).sum(axis=-1, dtype=np.float32)   # golden.py:51

    s_pre2 = h_pre - f32(hc_eps)                                # golden.py:53
    dh_pre2 = dh_pre * s_pre2 * (f32(1.0) - s_pre2)             # golden.py:54
    dh_post2 = dh_post * h_post * (f32(1.0) - h_post / f32(2))  # golden.py:55

    dh_pre1 = a_pre * dh_pre2                                   # golden.py:57-59
    dh_post1 = a_post * dh_post2
    dh_res1 = a_res * dh_res

    dh_mix_tmp = np.concatenate([dh_pre1, dh_post1, dh_res1.reshape(B, S, n * n)], axis=-1)  # :61
    dh_mix = dh_mix_tmp * inv_rms[:, :, None]                   # golden.py:62

    dvecX_mm = np.matmul(dh_mix, phi)                           # golden.py:65

    xrs = x_fp.reshape(T, nD) * gamma.reshape(1, nD)            # golden.py:68
    dphi = np.matmul(dh_mix.reshape(T, n * n + 2 * n).T, xrs)   # golden.py:69

    h_mix_tmp = h_mix * inv_rms[:, :, None]                     # golden.py:72-73
    h_pre1 = h_mix_tmp[..., :n]
    h_post1 = h_mix_tmp[..., n:2 * n]
    h_res1 = h_mix_tmp[..., 2 * n:]
    dinv_rms = (dh_mix_tmp * h_mix).sum(axis=-1, keepdims=True, dtype=np.float32)   # golden.py:74

    dalpha = np.array([(dh_pre2 * h_pre1).sum(dtype=np.float32),                   # golden.py:77-80
                       (dh_post2 * h_post1).sum(dtype=np.float32),
                       (dh_res.reshape(B, S, n * n) * h_res1).sum(dtype=np.float32)],
                      dtype=np.float32)

    dbias = np.concatenate([dh_pre2.sum(axis=(0, 1), dtype=np.float32),          # golden.py:83-86
                            dh_post2.sum(axis=(0, 1), dtype=np.float32),
                            dh_res.reshape(B, S, n * n).sum(axis=(0, 1), dtype=np.float32)])

    inv3 = inv_rms[:, :, None] ** 3                             # golden.py:89
    dvecX_inv = -(dinv_rms * inv3 / f32(nD)) * vecX
    dvecX_hin = h_pre[..., None] * h_in_fp_grad[:, :, None, :]  # golden.py:90
    dvecX_inv = dvecX_inv.reshape(B, S, n, D) + dvecX_hin       # golden.py:91

    dgamma = (x_fp.reshape(T, nD) * dvecX_mm.reshape(T, nD)).sum(axis=-2, dtype=np.float32)  # :93
    dx = dvecX_mm.reshape(B, S, n, D) * gamma.reshape(1, 1, n, D) + dvecX_inv   # golden.py:94

    return (f32_to_bf16(dx), dphi.astype(np.float32), dalpha,
            dbias.astype(np.float32), dgamma.astype(np.float32))   # golden.py:96


# ----------------------------------------------------------- tolerance helpers
def bf16_ulp(v: np.ndarray) -> np.ndarray:
    """Spacing of bf16 numbers at |v| (2^(e-7) for normals, 2^-133 floor)."""
    a = np.abs(np.asarray(v, dtype=np.float32))
    e = np.floor(np.log2(np.maximum(a, np.float32(2.0 ** -126))))
    return np.exp2(e - 7).astype(np.float32)


def forward_term_scale(x_bf16, h_pre):
    """Per-element sum of |terms| of h_in = sum_i h_pre[i] * x[i, :] (golden.py:62)."""
    x_f = bf16_to_f32(x_bf16)
    return (np.abs(np.asarray(h_pre, np.float32))[..., None] * np.abs(x_f)).sum(axis=2)


def backward_term_scale(x_bf16, phi, alpha, inv_rms, h_mix, h_pre, h_post,
                        dh_in_bf16, dh_post, dh_res, gamma, hc_eps=1e-6):
    """Per-element sum of |terms| that make up dx (src/backward/golden.py:65,89-94).

    |dh_mix| @ |phi| * |gamma| + |c * x| + |h_pre * dh_in|, with the scalar
    c = dinv_rms * inv_rms^3 / nD of golden.py:89.
    """
    B, S, n, D = x_bf16.shape
    nD = n * D
    f32 = np.float32
    x_fp = bf16_to_f32(x_bf16)
    dh = bf16_to_f32(dh_in_bf16)
    alpha = np.asarray(alpha, np.float32)
    h_pre = np.asarray(h_pre, np.float32)
    h_post = np.asarray(h_post, np.float32)
    inv_rms = np.asarray(inv_rms, np.float32)
    dh_pre = (dh[:, :, None, :] * x_fp).sum(axis=-1, dtype=np.float32)
    s = h_pre - f32(hc_eps)
    dh_pre2 = dh_pre * s * (f32(1) - s)
    dh_post2 = np.asarray(dh_post, np.float32) * h_post * (f32(1) - h_post / f32(2))
    tmp = np.concatenate([alpha[0] * dh_pre2, alpha[1] * dh_post2,
                          alpha[2] * np.asarray(dh_res, np.float32).reshape(B, S, n * n)], axis=-1)
    dh_mix = tmp * inv_rms[:, :, None]
    dinv = (tmp * np.asarray(h_mix, np.float32)).sum(axis=-1, keepdims=True)
    c = dinv * inv_rms[:, :, None] ** 3 / f32(nD)
    mm = np.matmul(np.abs(dh_mix), np.abs(np.asarray(phi, np.float32))).reshape(B, S, n, D)
    return (mm * np.abs(np.asarray(gamma, np.float32)).reshape(1, 1, n, D)
            + np.abs(c * x_fp.reshape(B, S, nD)).reshape(B, S, n, D)
            + np.abs(h_pre[..., None] * dh[:, :, None, :]))


def bf16_stats(ours_bf16, ref_bf16, term_scale, ulps=1.0, fp32_floor=2.0 ** -18) -> dict:
    """How far bf16 results are from the reference value, element by element.

    Keys: ``n`` elements; ``exact`` equal bit patterns (value-equal, so +0/-0
    count); ``within_ulp`` |ours - ref| <= ulps * ulp(ref) (exact included);
    ``floor_needed`` beyond that but within the fp32 accumulation floor
    ``fp32_floor * term_scale``; ``bad`` beyond both; ``worst_ulps`` the
    largest distance in ulps of ref; ``worst_ulps_no_floor`` the same over the
    elements that needed no floor (at most ``ulps`` when ``within_ulp`` holds
    everywhere else).
    """
    a = bf16_to_f32(ours_bf16)
    b = bf16_to_f32(ref_bf16)
    d = np.abs(a - b)
    u = bf16_ulp(b)
    in_ulp = d <= ulps * u
    floor = np.float32(fp32_floor) * np.asarray(term_scale, np.float32)
    ok = d <= ulps * u + floor
    dist = d / u
    return {
        "n": int(d.size),
        "exact": int((a == b).sum()),
        "within_ulp": int(in_ulp.sum()),
        "floor_needed": int((ok & ~in_ulp).sum()),
        "bad": int((~ok).sum()),
        "worst_ulps": float(dist.max()) if d.size else 0.0,
        "worst_ulps_no_floor": float(dist[in_ulp].max()) if in_ulp.any() else 0.0,
    }


def bf16_within(ours_bf16, ref_bf16, term_scale, ulps=1.0, fp32_floor=2.0 ** -18):
    """Elementwise check |ours - ref| <= ulps * ulp(ref) + fp32_floor * term_scale.

    The second term is the fp32 accumulation bound: two fp32 summation orders
    of the same terms may differ by a few 2^-24 * sum|terms|, which is many bf16
    ulps of a result produced by cancellation.  Returns (ok, worst_ulps, n_bad).
    """
    st = bf16_stats(ours_bf16, ref_bf16, term_scale, ulps, fp32_floor)
    return st["bad"] == 0, st["worst_ulps"], st["bad"]
