"""Token-sharded data parallelism, host logic, on CPU ranks (gloo, world size 2).

The CUDA kernels are replaced by the CPU oracle here (the injected fwd/bwd of
DataParallelMHC), so what is tested is the sharding, the flat gradient buffer
and the all-reduce: the summed per-shard gradients must equal the full-batch
gradients.  A second test kills one rank before the all-reduce and checks
that the survivor gets an error within the process-group timeout instead of
waiting forever.
"""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mhc_ops_b200.backward import param_grad_numel, split_param_grads
from mhc_ops_b200.dist import DataParallelMHC, shard_bounds, shard_tokens
from mhc_ops_b200.synthetic import make_inputs


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _oracle_fwd(x, phi, alpha, bias, outflag=True, **kw):
    from oracle import mhc_oracle as O
    out = O.forward(_bits(x), phi.numpy(), alpha.numpy(), bias.numpy(), outflag=True)
    h_in = torch.from_numpy(out[0].view(np.int16).copy()).view(torch.bfloat16)
    return (h_in,) + tuple(torch.from_numpy(np.ascontiguousarray(o)) for o in out[1:])


def _oracle_bwd(x, phi, alpha, bias, inv_rms, h_mix, h_pre, h_post, dh_in, dh_post, dh_res, gamma,
                grad_out=None, **kw):
    from oracle import mhc_oracle as O
    dx, dphi, dalpha, dbias, dgamma = O.backward(
        _bits(x), phi.numpy(), alpha.numpy(), bias.numpy(), inv_rms.numpy(), h_mix.numpy(), h_pre.numpy(),
        h_post.numpy(), _bits(dh_in), dh_post.numpy(), dh_res.numpy(), gamma.numpy())
    n, D = x.shape[2], x.shape[3]
    views = split_param_grads(grad_out, n, D)
    for v, src in zip(views, (dphi, dgamma, dalpha, dbias)):
        v.copy_(torch.from_numpy(np.ascontiguousarray(src)).reshape(v.shape))
    dx_t = torch.from_numpy(dx.view(np.int16).copy()).view(torch.bfloat16)
    return dx_t, views[0], views[2], views[3], views[1]


def _worker_allreduce(rank, world, port, q, overlap=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        # a generous rendezvous limit: a rank's first `import torch` in a fresh
        # container can take a minute
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=180))
    except Exception:   # noqa: BLE001 - reported to the test, which may retry on another port
        q.put((rank, "rendezvous", traceback.format_exc()))
        return
    try:
        inp = make_inputs(2, 9, 4, 32, seed=7)   # 18 tokens: uneven split is fine too
        sh = {k: shard_tokens(getattr(inp, k), rank, world) for k in ("x", "dh_in", "dh_post", "dh_res")}
        dp = DataParallelMHC(4, 32, fwd=_oracle_fwd, bwd=_oracle_bwd)
        h_in, h_post, h_res, inv_rms, h_mix, h_pre = dp.forward(sh["x"], inp.phi, inp.alpha, inp.bias)
        dx, dphi, dalpha, dbias, dgamma = dp.backward(sh["x"], inp.phi, inp.alpha, inp.bias, inv_rms, h_mix,
                                                      h_pre, h_post, sh["dh_in"], sh["dh_post"], sh["dh_res"],
                                                      inp.gamma, overlap=overlap)
        dp.wait()   # with overlap the all-reduce was left in flight
        q.put((rank, "ok", (dphi.clone(), dalpha.clone(), dbias.clone(), dgamma.clone(), dx.clone())))
    except Exception:   # noqa: BLE001 - reported to the test with its traceback
        q.put((rank, "error", traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def _worker_dies(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # rendezvous with a generous limit (slow first imports), then a group whose
    # collectives give up after 5 s: the survivor's error comes from that limit
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=180))
    group = dist.new_group(ranks=list(range(world)), timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)          # the failing rank leaves between steps, before the collective
    flat = torch.ones(param_grad_numel(4, 8))
    try:
        dist.all_reduce(flat, group=group)
        q.put((rank, "no error"))
    except Exception as e:   # noqa: BLE001 - any collective error is the detection we want
        q.put((rank, f"error: {type(e).__name__}"))


def test_shard_bounds_cover_all_tokens_once():
    for T in (0, 1, 7, 18, 4096):
        for w in (1, 2, 3, 4, 8):
            spans = [shard_bounds(T, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == T
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1


def _run_allreduce_ranks(world, overlap):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_allreduce, args=(r, world, port, q, overlap)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(results, key=lambda r: r[0]), [p.exitcode for p in procs]


@pytest.mark.parametrize("overlap", [False, True])
def test_allreduced_shard_grads_equal_full_batch_grads(overlap):
    world = 2
    results, codes = _run_allreduce_ranks(world, overlap)
    if any(r[1] == "rendezvous" for r in results):
        # the port picked for the store was taken before rank 0 bound it: once more on another
        results, codes = _run_allreduce_ranks(world, overlap)
    for r in results:
        assert r[1] == "ok", f"rank {r[0]}: {r[1]}\n{r[2]}"
    assert codes == [0] * world, codes
    results = [(r[0],) + r[2] for r in results]

    inp = make_inputs(2, 9, 4, 32, seed=7)
    full = _oracle_fwd(inp.x, inp.phi, inp.alpha, inp.bias)
    flat = torch.empty(param_grad_numel(4, 32))
    dx, dphi, dalpha, dbias, dgamma = _oracle_bwd(inp.x, inp.phi, inp.alpha, inp.bias, *full[3:5], full[5],
                                                  full[1], inp.dh_in, inp.dh_post, inp.dh_res, inp.gamma,
                                                  grad_out=flat)
    for _, g_phi, g_alpha, g_bias, g_gamma, _dx in results:
        for got, ref in ((g_phi, dphi), (g_alpha, dalpha), (g_bias, dbias), (g_gamma, dgamma)):
            assert (got - ref).abs().max() <= 1e-5 * ref.abs().max()
    dx_cat = torch.cat([r[5].reshape(-1, 4, 32) for r in results], 0)
    assert torch.equal(dx_cat, dx.reshape(-1, 4, 32))


def test_dead_rank_is_detected_by_collective_timeout():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_dies, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    rank, msg = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and msg.startswith("error"), msg
    assert procs[1].exitcode == 3
