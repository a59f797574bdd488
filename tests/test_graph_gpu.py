"""The pre-op inside CUDA graphs: a training or serving loop captures one
step (forward with the outflag outputs, then the backward) once and replays
it with new inputs copied into the same buffers.  The captured kernels take
their tensor maps and workspace pointers by value, so a replay must equal an
eager call on the same inputs bit for bit.  The workspace has to exist before
the capture (nothing is allocated or synchronised while a stream captures):
one call on the capturing stream first, as torch's own warm-up advice says;
without it the call raises a clear error instead of a CUDA failure.
"""
import pytest
import torch

from mhc_ops_b200 import mhc_backward_manual, mhc_forward_pre, ops
from mhc_ops_b200.synthetic import make_inputs

# (B, S, n, D): fused tensor-core forward + n = 4 tensor-core backward;
# two-kernel forward + tiled backward (n = 8); generic kernels (D = 100)
SHAPES = ((2, 1024, 4, 4096), (1, 300, 8, 1024), (1, 77, 3, 100))


def _step_api(t):
    fw = mhc_forward_pre(t["x"], t["phi"], t["alpha"], t["bias"], outflag=True)
    bw = mhc_backward_manual(t["x"], t["phi"], t["alpha"], t["bias"], fw[3], fw[4], fw[5], fw[1], t["dh_in"],
                             t["dh_post"], t["dh_res"], t["gamma"])
    return tuple(fw) + tuple(bw)


def _step_ops(t):
    fw = ops.fwd(t["x"], t["phi"], t["alpha"], t["bias"])
    bw = ops.bwd(t["x"], t["phi"], t["alpha"], fw[3], fw[4], fw[5], fw[1], t["dh_in"], t["dh_post"], t["dh_res"],
                 t["gamma"])
    return tuple(fw) + tuple(bw)


def _tensors(B, S, n, D, seed):
    d = make_inputs(B, S, n, D, seed=seed).to("cuda")
    return {k: getattr(d, k).clone() for k in ("x", "phi", "alpha", "bias", "dh_in", "dh_post", "dh_res", "gamma")}


@pytest.mark.gpu
@pytest.mark.parametrize("step", [_step_api, _step_ops], ids=["python-api", "torch-ops"])
@pytest.mark.parametrize("B,S,n,D", SHAPES)
def test_replayed_step_equals_eager(step, B, S, n, D):
    static = _tensors(B, S, n, D, seed=71)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step(static)                       # warm-up: the workspace of stream s
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        outs = step(static)
    for seed in (72, 73):                  # new inputs in the captured buffers, then replay
        fresh = _tensors(B, S, n, D, seed=seed)
        for k, v in fresh.items():
            static[k].copy_(v)
        g.replay()
        torch.cuda.synchronize()
        ref = step(fresh)
        torch.cuda.synchronize()
        for i, (a, b) in enumerate(zip(outs, ref)):
            assert a.shape == b.shape and a.dtype == b.dtype, i
            assert torch.equal(a.view(torch.uint8) if a.dtype == torch.bfloat16 else a,
                               b.view(torch.uint8) if b.dtype == torch.bfloat16 else b), \
                f"output {i}: replay differs from the eager call (seed {seed})"
    del g


@pytest.mark.gpu
@pytest.mark.parametrize("step", [_step_api, _step_ops], ids=["python-api", "torch-ops"])
def test_capture_without_a_workspace_raises(step):
    t = _tensors(1, 64, 4, 256, seed=74)
    s = torch.cuda.Stream()               # never used before: no workspace yet
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with pytest.raises(RuntimeError, match="capturing a CUDA graph"):
        with torch.cuda.graph(g, stream=s):
            step(t)
    del g
    torch.cuda.synchronize()
