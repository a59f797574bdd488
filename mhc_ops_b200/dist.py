"""Token-sharded data parallelism for the mHC pre-op.

The op is per-token: the forward needs no communication and the backward's
dx is local.  Only the parameter gradients (dphi [N,nD], dgamma [nD],
dalpha [3], dbias [N]) are sums over tokens, so each rank runs the backward
on its token shard into one flat fp32 buffer and a single all-reduce (SUM)
of that buffer -- NCCL over NVLink on GPUs, gloo on CPU -- produces the
global gradients.  The reference has no multi-process path; this is new.

Determinism: each rank's local reduction has a fixed order, and the
all-reduce runs over a fixed rank count, so results are reproducible for a
given world size.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .backward import param_grad_numel, split_param_grads

__all__ = ["shard_bounds", "shard_tokens", "allreduce_param_grads", "DataParallelMHC"]


def shard_bounds(tokens: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) token range of `rank` (first ranks take the remainder)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, rem = divmod(tokens, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def shard_tokens(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank's contiguous share of the flattened (B*S) token axis of a [B,S,...] tensor,
    returned as [1, tokens_of_rank, ...]."""
    B, S = t.shape[0], t.shape[1]
    flat = t.reshape(B * S, *t.shape[2:])
    a, b = shard_bounds(B * S, rank, world)
    return flat[a:b].unsqueeze(0)


def allreduce_param_grads(flat: torch.Tensor, group=None, async_op: bool = False):
    """SUM-all-reduce the flat [dphi | dgamma | dalpha | dbias] buffer in place."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return None
    return dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group, async_op=async_op)


class DataParallelMHC:
    """Runs forward/backward on this rank's token shard and all-reduces the param grads.

    ``backward(...)`` returns (dx_local, dphi, dalpha, dbias, dgamma) with the
    parameter gradients summed over all ranks (views into one flat buffer).
    ``fwd`` / ``bwd`` are the forward and backward callables (the CUDA ones by
    default); tests inject others to exercise the host logic on CPU ranks.
    """

    def __init__(self, n: int, D: int, group=None, fwd=None, bwd=None, device=None):
        self.n, self.D, self.group = n, D, group
        if fwd is None or bwd is None:
            from .backward import mhc_backward_manual
            from .forward import mhc_forward_pre
            fwd = fwd or mhc_forward_pre
            bwd = bwd or mhc_backward_manual
        self.fwd, self.bwd = fwd, bwd
        self.device = device
        self.flat = None
        self.pending = None   # all-reduce still in flight (backward(..., overlap=True))

    def grad_buffer(self, device) -> torch.Tensor:
        numel = param_grad_numel(self.n, self.D)
        if self.flat is None or self.flat.device != torch.device(device) or self.flat.numel() != numel:
            self.flat = torch.empty(numel, dtype=torch.float32, device=device)
        return self.flat

    def forward(self, x, phi, alpha, bias, **kw):
        return self.fwd(x, phi, alpha, bias, outflag=True, **kw)

    def backward(self, x, phi, alpha, bias, inv_rms, h_mix, h_pre, h_post, dh_in, dh_post, dh_res, gamma,
                 overlap: bool = False, **kw):
        """Returns ``(dx_local, dphi, dalpha, dbias, dgamma)``.

        The four parameter gradients are views into one flat buffer owned by
        this object, which every ``backward`` call rewrites.  With
        ``overlap=False`` they hold the sums over all ranks when this returns
        (in stream order).  With ``overlap=True`` the all-reduce is left in
        flight on NCCL's own stream so that whatever the caller enqueues next
        -- typically the next step's forward -- overlaps it: the views then
        hold this rank's partial sums until ``wait()`` has been called, and
        reading them before that gives partial or mixed values.  The next
        ``backward`` calls ``wait()`` itself and then overwrites the buffer, so
        a caller that keeps the gradients across steps must ``wait()`` and
        copy them first."""
        self.wait()
        flat = self.grad_buffer(x.device)
        dx, dphi, dalpha, dbias, dgamma = self.bwd(x, phi, alpha, bias, inv_rms, h_mix, h_pre, h_post,
                                                   dh_in, dh_post, dh_res, gamma, grad_out=flat, **kw)
        work = allreduce_param_grads(flat, self.group, async_op=overlap)
        if overlap:
            self.pending = work
        dphi, dgamma, dalpha, dbias = split_param_grads(flat, self.n, self.D)
        return dx, dphi, dalpha, dbias, dgamma

    def wait(self):
        """Order the current stream after an all-reduce left in flight (no host wait for NCCL)."""
        if self.pending is not None:
            self.pending.wait()
            self.pending = None
