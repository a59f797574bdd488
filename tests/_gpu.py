"""Helpers for the GPU parity tests: run the CUDA path and the CPU oracle on the same bytes."""
import numpy as np
import torch

from oracle import mhc_oracle as O

FP32_TOL = 1e-4   # fp32 outputs: max|a-b| / max|ref|
DEV = "cuda:0"
# bf16 outputs (h_in, dx): within 1 ulp of the reference value, or, for at
# most this fraction of the elements (values produced by cancellation), within
# the fp32 accumulation floor 2^-18 * sum|terms|.
FLOOR_FRAC = 1e-3

# (tag, tensor, stats) of every bf16 comparison, printed at the end of the run
BF16_REPORT: list = []


def check_bf16(tag: str, name: str, ours_bits, ref_bits, scale) -> dict:
    """Compare bf16 outputs with the reference value; record and assert.

    Every element must be within 1 ulp + 2^-18 * sum|terms|; the elements that
    needed the second term (beyond 1 ulp) are counted, reported at the end of
    the run with the worst ulp distance, and bounded by FLOOR_FRAC.
    """
    st = O.bf16_stats(ours_bits, ref_bits, scale)
    BF16_REPORT.append((tag, name, st))
    assert st["bad"] == 0, f"{tag} {name}: {st['bad']} elements beyond tolerance ({st})"
    assert st["floor_needed"] <= FLOOR_FRAC * st["n"] + 8, f"{tag} {name}: too many need the fp32 floor ({st})"
    return st


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
    check_bf16(tag, "h_in", bits(out[0]), ref[0], O.forward_term_scale(x_bits, ref[5]))


def assert_bwd_close(out, ref, scale, tag=""):
    names = ("dx", "dphi", "dalpha", "dbias", "dgamma")
    for nm, o, r in zip(names[1:], out[1:], ref[1:]):
        assert tuple(o.shape) == tuple(np.shape(r)), (tag, nm)
        e = rel(o, r)
        assert e <= FP32_TOL, f"{tag} {nm}: rel err {e:.3g}"
    check_bf16(tag, "dx", bits(out[0]), ref[0], scale)


def _oracle_shard_worker(job):
    """One token shard checked against the oracle in a worker process: the
    forward from x, the backward from the GPU's forward intermediates (so
    both backward implementations see the same inputs).  Returns the fp32
    relative errors, the bf16 statistics and the shard's parameter gradients."""
    (xs, dhs, dpost, dres, phi, alpha, bias, gamma, h_in_b, f_np, dx_b) = job
    ref = O.forward(xs, phi, alpha, bias, outflag=True)
    res = {"fwd_rel": {}, "param": None}
    for nm, o, r in zip(("h_post", "h_res", "inv_rms", "h_mix", "h_pre"), f_np, ref[1:]):
        res["fwd_rel"][nm] = rel(o, r)
    res["h_in"] = O.bf16_stats(h_in_b, ref[0], O.forward_term_scale(xs, ref[5]))
    h_post, _, inv_rms, h_mix, h_pre = f_np
    rb = O.backward(xs, phi, alpha, bias, inv_rms, h_mix, h_pre, h_post, dhs, dpost, dres, gamma)
    scale = O.backward_term_scale(xs, phi, alpha, inv_rms, h_mix, h_pre, h_post, dhs, dpost, dres, gamma)
    res["dx"] = O.bf16_stats(dx_b, rb[0], scale)
    res["param"] = tuple(np.asarray(r, np.float64) for r in rb[1:])
    return res


def oracle_shards(jobs, workers=None):
    """Run _oracle_shard_worker over the jobs in a spawn pool (this process
    holds a CUDA context, so no fork), BLAS threads split over the workers."""
    import concurrent.futures as cf
    import multiprocessing as mp
    import os
    cores = os.cpu_count() or 1
    workers = max(1, min(workers or max(1, cores // 2), len(jobs)))
    keep = {k: os.environ.get(k) for k in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")}
    for k in keep:
        os.environ[k] = str(max(1, cores // workers))
    try:
        with cf.ProcessPoolExecutor(workers, mp_context=mp.get_context("spawn")) as ex:
            return list(ex.map(_oracle_shard_worker, jobs))
    finally:
        for k, v in keep.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
