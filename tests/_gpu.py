"""Helpers for the GPU parity tests: run the CUDA path and the CPU oracle on the same bytes."""
import numpy as np
import torch

from oracle import mhc_oracle as O

FP32_TOL = 1e-4   # fp32 outputs: max|a-b| / max|ref|
DEV = "cuda:0"


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_bits(a: np.ndarray, device=DEV) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16).copy()).view(torch.bfloat16).to(device)


def rel(a, b) -> float:
    a = a.detach().float().cpu().numpy() if torch.is_tensor(a) else np.asarray(a, np.float32)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)) if b.size else 0.0


def assert_fwd_close(out, ref, x_bits, tag=""):
    """out: CUDA outputs (6-tuple); ref: oracle/golden outputs (numpy 6-tuple)."""
    names = ("h_in", "h_post", "h_res", "inv_rms", "h_mix", "h_pre")
    for nm, o, r in zip(names[1:], out[1:], ref[1:]):
        assert tuple(o.shape) == tuple(r.shape), (tag, nm)
        e = rel(o, r)
        assert e <= FP32_TOL, f"{tag} {nm}: rel err {e:.3g}"
    ok, worst, nbad = O.bf16_within(bits(out[0]), ref[0], O.forward_term_scale(x_bits, ref[5]))
    assert ok, f"{tag} h_in: {nbad} elements beyond tolerance (worst {worst:.1f} ulp)"


def assert_bwd_close(out, ref, scale, tag=""):
    names = ("dx", "dphi", "dalpha", "dbias", "dgamma")
    for nm, o, r in zip(names[1:], out[1:], ref[1:]):
        assert tuple(o.shape) == tuple(np.shape(r)), (tag, nm)
        e = rel(o, r)
        assert e <= FP32_TOL, f"{tag} {nm}: rel err {e:.3g}"
    ok, worst, nbad = O.bf16_within(bits(out[0]), ref[0], scale)
    assert ok, f"{tag} dx: {nbad} elements beyond tolerance (worst {worst:.1f} ulp)"
