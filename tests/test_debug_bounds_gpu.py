"""The debug-bounds build (-DMHC_DEBUG_BOUNDS, lib/libmhc_ops_dbg.so).

Every checked global access of its kernels must fall inside the buffers the
entry point was called with; one that does not is skipped and recorded, and
nothing traps.  A child process runs the odd-shape cases of
tests/_bounds_cases.py on that library and checks the record after every
call; this process runs the same cases on the normal library, and the outputs
must agree bit for bit (the checks change no arithmetic).  The child also runs
mhc_debug_bounds_selftest, whose kernel checks an address one byte past the
one buffer it registered, without reading it, so the record path itself is
seen to work.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.gpu
def test_debug_bounds_build_sees_no_out_of_buffer_access_and_matches_normal_build(tmp_path):
    from mhc_ops_b200 import build

    dbg = build.build(debug_bounds=True)
    out = str(tmp_path / "dbg.npz")
    env = dict(os.environ, MHC_OPS_LIBRARY=dbg, PYTHONPATH=ROOT)
    res = subprocess.run([sys.executable, "-m", "tests._bounds_cases", out], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, f"debug-bounds run failed:\n{res.stdout[-3000:]}\n{res.stderr[-3000:]}"
    got = dict(np.load(out))

    count, site, offset, nbytes = (int(v) for v in got.pop("selftest"))
    assert count == 1 and offset == 256 and nbytes == 1, (count, site, offset, nbytes)
    assert site // 100000 == 7, f"self-test site {site} is not in mhc_ops.cu"

    from tests._bounds_cases import run_cases
    ref = run_cases(debug=False)
    assert set(ref) == set(got), sorted(set(ref) ^ set(got))
    for k in ref:
        assert ref[k].dtype == got[k].dtype and ref[k].shape == got[k].shape, k
        same = ref[k].view(np.uint8) == got[k].view(np.uint8)
        assert same.all(), f"{k}: debug-bounds build differs in {int((~same).sum())} of {same.size} bytes"
    torch.cuda.synchronize()
