"""Generate the golden fixtures under tests/golden/ by running the REFERENCE golden.

The reference (folrent1896/mhc_ops) is a Python/PyTorch package; its golden
forward ``src/forward/golden.py:mhc_forward_pre`` and golden backward
``src/backward/golden.py:mhc_backward_manual`` are imported here straight from
their files (no Triton import), run on the CPU on seeded inputs, and the
inputs plus every output are stored as ``<case>.npz`` (bf16 as uint16 bits).

The reference checkout is only available where the fixtures are generated;
the committed ``.npz`` files are what the tests read.  Its location is
required: ``--reference <checkout>`` or the ``MHC_REFERENCE_ROOT``
environment variable.

Usage:  python tests/golden/make_golden.py --reference <path to the reference checkout>
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from mhc_ops_b200.synthetic import make_inputs  # noqa: E402

# (name, B, S, n, D, convention, seed, phi_scale, with_backward)
CASES = [
    # the golden-forward case: B=2,S=128,n=4,D=256, phi ~ N(0,1) unscaled.
    ("fwd_cfg1_2x128x4x256", 2, 128, 4, 256, "standard", 0, 1.0, True),
    # The reference's own backward test: test/backward/test_backward.py:44-65 (seeds 42/123).
    ("refconv_2x64x4x128", 2, 64, 4, 128, "reference", 42, None, True),
    # README backward shape family with the fan-in scaled phi and gamma ~ 1 + 0.1 N(0,1).
    ("bwd_2x64x4x256", 2, 64, 4, 256, "standard", 1, None, True),
    # Wider hyper-connection n=8 (N = 80).
    ("n8_1x64x8x128", 1, 64, 8, 128, "standard", 2, None, True),
    # quick_test.py:194 tiny printout shape B=1,S=2,n=2,D=4.
    ("tiny_1x2x2x4", 1, 2, 2, 4, "reference", 42, None, True),
    # Ragged: prime token count, D not a multiple of 128.
    ("ragged_1x7x4x64", 1, 7, 4, 64, "standard", 3, None, True),
]


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MHC_REFERENCE_ROOT"),
                    help="root of the reference checkout (default: $MHC_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <checkout root> or set MHC_REFERENCE_ROOT")
    fwd_mod = _load(os.path.join(args.reference, "src/forward/golden.py"), "ref_fwd_golden")
    bwd_mod = _load(os.path.join(args.reference, "src/backward/golden.py"), "ref_bwd_golden")
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    for name, B, S, n, D, conv, seed, scale, with_bwd in CASES:
        inp = make_inputs(B, S, n, D, seed=seed, phi_scale=scale, convention=conv)
        with torch.no_grad():
            h_in, h_post, h_res, inv_rms, h_mix, h_pre = fwd_mod.mhc_forward_pre(
                inp.x, inp.phi, inp.alpha, inp.bias, outflag=True)
            rec = dict(
                shape=np.array([B, S, n, D], dtype=np.int64),
                x=_bits(inp.x), phi=inp.phi.numpy(), alpha=inp.alpha.numpy(), bias=inp.bias.numpy(),
                gamma=inp.gamma.numpy(), dh_in=_bits(inp.dh_in), dh_post=inp.dh_post.numpy(),
                dh_res=inp.dh_res.numpy(),
                h_in=_bits(h_in), h_post=h_post.numpy(), h_res=h_res.numpy(),
                inv_rms=inv_rms.numpy(), h_mix=h_mix.numpy(), h_pre=h_pre.numpy(),
            )
            if with_bwd:
                dx, dphi, dalpha, dbias, dgamma = bwd_mod.mhc_backward_manual(
                    inp.x, inp.phi, inp.alpha, inp.bias, inv_rms, h_mix, h_pre, h_post,
                    inp.dh_in, inp.dh_post, inp.dh_res, inp.gamma)
                rec.update(dx=_bits(dx), dphi=dphi.numpy(), dalpha=dalpha.numpy(),
                           dbias=dbias.numpy(), dgamma=dgamma.numpy())
        out = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(out, **rec)
        print(f"wrote {out} ({os.path.getsize(out) / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
