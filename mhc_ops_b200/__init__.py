"""mhc_ops_b200 -- B200 (sm_100a) implementation of the mHC pre-op of folrent1896/mhc_ops.

Mirrors the reference package facade (``src/__init__.py:13-48``): the golden
and the Triton names resolve to the same CUDA kernels here, reached through the
C ABI of ``lib/libmhc_ops.so`` (``include/mhc_ops.h``).  Adds the autograd
wrapper ``MHCPreFunction`` / ``mhc_pre``, the post-op that consumes
``h_post`` / ``h_res`` (``mhc_post``, ``MHCPostFunction``; absent from the
reference) and token-sharded data parallelism (``mhc_ops_b200.dist``).
TileLang names of the reference are not provided (the reference's TileLang
code does not run).
"""

__version__ = "0.2.0"

from .forward import (mhc_forward_pre, mhc_forward_pre_fp8, mhc_forward_pre_fused_norm,  # noqa: E402
                      mhc_forward_pre_triton, mhc_forward_pre_triton_optimized, quantize_fp8_pow2)
from .backward import mhc_backward_manual, mhc_backward_triton  # noqa: E402
from .autograd import MHCPreFunction, mhc_pre  # noqa: E402
from .post import MHCPostFunction, mhc_post, mhc_post_backward, mhc_post_fn  # noqa: E402

__all__ = [
    "mhc_forward_pre",
    "mhc_forward_pre_triton",
    "mhc_forward_pre_triton_optimized",
    "mhc_forward_pre_fused_norm",
    "mhc_forward_pre_fp8",
    "quantize_fp8_pow2",
    "mhc_backward_manual",
    "mhc_backward_triton",
    "MHCPreFunction",
    "mhc_pre",
    "mhc_post",
    "mhc_post_backward",
    "MHCPostFunction",
    "mhc_post_fn",
]
