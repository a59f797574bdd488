"""Seeded synthetic inputs for the mHC pre-op.

Two draw orders are provided; both use the CPU torch generator so that every
consumer (the CUDA path, the CPU oracle, the bench) sees identical bytes.

``convention="standard"`` (default)
    ``torch.manual_seed(seed)`` then, in order: ``x ~ N(0,1)`` bf16
    ``[B,S,n,D]``; ``phi ~ N(0,1) * phi_scale`` fp32 ``[N,nD]`` (``phi_scale``
    defaults to ``1/sqrt(nD)``); ``alpha = [1.1, 0.9, 1.05]``;
    ``bias ~ 0.1 N(0,1)`` ``[N]``; ``gamma ~ 1 + 0.1 N(0,1)`` ``[n,D]``;
    ``dh_in ~ N(0,1)`` bf16 ``[B,S,D]``; ``dh_post ~ N(0,1)`` ``[B,S,n]``;
    ``dh_res ~ N(0,1)`` ``[B,S,n,n]``.

``convention="reference"``
    The draw order of the reference's own tests
    (``test/backward/test_backward.py:44-65``, ``test/backward/benchmark.py:132-155``):
    ``manual_seed(seed)`` (42 there) for ``x, phi (unscaled), bias, gamma ~ N(0,1)``,
    then ``manual_seed(grad_seed)`` (123 there) for ``dh_in, dh_post, dh_res``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


def n_out(n: int) -> int:
    return n * n + 2 * n


@dataclass
class MhcInputs:
    x: torch.Tensor        # bf16 [B,S,n,D]
    phi: torch.Tensor      # fp32 [N,nD]
    alpha: torch.Tensor    # fp32 [3]
    bias: torch.Tensor     # fp32 [N]
    gamma: torch.Tensor    # fp32 [n,D]
    dh_in: torch.Tensor    # bf16 [B,S,D]
    dh_post: torch.Tensor  # fp32 [B,S,n]
    dh_res: torch.Tensor   # fp32 [B,S,n,n]

    def to(self, device) -> "MhcInputs":
        return MhcInputs(**{k: getattr(self, k).to(device) for k in self.__dataclass_fields__})

    @property
    def shape(self):
        return tuple(self.x.shape)


def make_inputs(B: int, S: int, n: int, D: int, seed: int = 0, phi_scale: float | None = None,
                convention: str = "standard", grad_seed: int = 123) -> MhcInputs:
    """Draw one seeded input set on the CPU (see module docstring for the order)."""
    N = n_out(n)
    nD = n * D
    if convention == "standard":
        if phi_scale is None:
            phi_scale = 1.0 / math.sqrt(nD)
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(B, S, n, D, generator=g, dtype=torch.bfloat16)
        phi = torch.randn(N, nD, generator=g, dtype=torch.float32) * phi_scale
        alpha = torch.tensor([1.1, 0.9, 1.05], dtype=torch.float32)
        bias = torch.randn(N, generator=g, dtype=torch.float32) * 0.1
        gamma = 1.0 + 0.1 * torch.randn(n, D, generator=g, dtype=torch.float32)
        dh_in = torch.randn(B, S, D, generator=g, dtype=torch.bfloat16)
        dh_post = torch.randn(B, S, n, generator=g, dtype=torch.float32)
        dh_res = torch.randn(B, S, n, n, generator=g, dtype=torch.float32)
    elif convention == "reference":
        torch.manual_seed(seed)
        x = torch.randn(B, S, n, D, dtype=torch.bfloat16)
        phi = torch.randn(N, nD, dtype=torch.float32)
        if phi_scale is not None:
            phi = phi * phi_scale
        alpha = torch.tensor([1.1, 0.9, 1.05], dtype=torch.float32)
        bias = torch.randn(N, dtype=torch.float32) * 0.1
        gamma = torch.randn(n, D, dtype=torch.float32)
        torch.manual_seed(grad_seed)
        dh_in = torch.randn(B, S, D, dtype=torch.bfloat16)
        dh_post = torch.randn(B, S, n, dtype=torch.float32)
        dh_res = torch.randn(B, S, n, n, dtype=torch.float32)
    else:
        raise ValueError(f"unknown convention {convention!r}")
    return MhcInputs(x, phi, alpha, bias, gamma, dh_in, dh_post, dh_res)
