"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, the ctypes mirrors of the argument structs match the C
layout, and host-side validation answers without touching a device."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest
import torch

from mhc_ops_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mhc_ops.h")


def _declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^MHC_API[^(]*?\b(mhc_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from mhc_ops_b200 import build
    build.build()
    return _lib.load()


def test_header_declares_the_api():
    syms = _declared_symbols()
    assert {"mhc_fwd", "mhc_bwd", "mhc_fwd_workspace_size", "mhc_bwd_workspace_size"} <= set(syms)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.lib_path()], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (mhc_\w+)$", out, flags=re.M))
    missing = [s for s in _declared_symbols() if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    for s in _declared_symbols():
        assert hasattr(lib, s)
    assert set(_lib.SIGNATURES) == set(_declared_symbols())


def test_ctypes_structs_match_c_layout():
    src = r'''
#include <stdio.h>
#include <stddef.h>
#include "mhc_ops.h"
#define F(s, m) printf(#s "." #m " %zu\n", offsetof(s, m));
int main(void) {
  printf("mhc_fwd_args %zu\n", sizeof(mhc_fwd_args));
  printf("mhc_bwd_args %zu\n", sizeof(mhc_bwd_args));
  F(mhc_fwd_args, tokens) F(mhc_fwd_args, n) F(mhc_fwd_args, D) F(mhc_fwd_args, norm_eps)
  F(mhc_fwd_args, workspace) F(mhc_fwd_args, workspace_bytes)
  F(mhc_bwd_args, dgamma) F(mhc_bwd_args, tokens) F(mhc_bwd_args, hc_eps) F(mhc_bwd_args, workspace_bytes)
  printf("mhc_post_fwd_args %zu\n", sizeof(mhc_post_fwd_args));
  printf("mhc_post_bwd_args %zu\n", sizeof(mhc_post_bwd_args));
  F(mhc_post_fwd_args, out) F(mhc_post_fwd_args, tokens) F(mhc_post_fwd_args, D)
  F(mhc_post_bwd_args, dh_post) F(mhc_post_bwd_args, tokens) F(mhc_post_bwd_args, D)
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "layout.c")
        exe = os.path.join(d, "layout")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-std=c99", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        lines = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.split() for l in lines if l.strip())
    classes = {"mhc_fwd_args": _lib.FwdArgs, "mhc_bwd_args": _lib.BwdArgs,
               "mhc_post_fwd_args": _lib.PostFwdArgs, "mhc_post_bwd_args": _lib.PostBwdArgs}
    for sname, cls in classes.items():
        assert int(got[sname]) == ctypes.sizeof(cls), sname
    for key, val in got.items():
        if "." in key:
            sname, field = key.split(".")
            assert getattr(classes[sname], field).offset == int(val), key


def test_status_strings_and_version(lib):
    assert lib.mhc_abi_version() == 10400
    assert lib.mhc_status_string(0) == b"ok"
    for code in range(1, 11):
        assert lib.mhc_status_string(code) != b"unknown mhc status"
    assert lib.mhc_status_string(99) == b"unknown mhc status"


def test_fwd_workspace_size_validates_shapes_without_a_device(lib):
    out = ctypes.c_size_t(0)
    assert lib.mhc_fwd_workspace_size(16, 4, 64, ctypes.byref(out)) == 0 and out.value >= 256
    assert lib.mhc_fwd_workspace_size(16, 9, 64, ctypes.byref(out)) == 2      # n > 8
    assert lib.mhc_fwd_workspace_size(-1, 4, 64, ctypes.byref(out)) == 2      # T < 0
    assert lib.mhc_fwd_workspace_size(16, 4, 0, ctypes.byref(out)) == 2       # D < 1
    assert lib.mhc_fwd_workspace_size(16, 4, 64, None) == 1                   # NULL out


def test_null_args_rejected(lib):
    assert lib.mhc_fwd(None, None) == 1
    assert lib.mhc_bwd(None, None) == 1


def test_cpu_tensors_raise_no_fallback():
    from mhc_ops_b200 import mhc_backward_manual, mhc_forward_pre
    from mhc_ops_b200.synthetic import make_inputs
    i = make_inputs(1, 2, 4, 8)
    with pytest.raises(RuntimeError, match="CUDA only"):
        mhc_forward_pre(i.x, i.phi, i.alpha, i.bias)
    with pytest.raises(RuntimeError, match="CUDA only"):
        mhc_backward_manual(i.x, i.phi, i.alpha, i.bias, torch.ones(1, 2), torch.zeros(1, 2, 24),
                            torch.ones(1, 2, 4), torch.ones(1, 2, 4), i.dh_in, i.dh_post, i.dh_res, i.gamma)


def test_product_path_does_not_import_the_oracle():
    pkg = os.path.join(ROOT, "mhc_ops_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh")):
                text = open(os.path.join(dirpath, f)).read()
                assert not re.search(r"(import\s+oracle|from\s+oracle|mhc_oracle)", text), f


def test_c_program_links_the_library_and_agrees_with_ctypes():
    """A plain C caller (the native boundary, not ctypes) links libmhc_ops.so and
    gets the same device-free answers as the Python binding."""
    src = r'''
#include <stdio.h>
#include "mhc_ops.h"
int main(void) {
  size_t fw = 0, bw = 0;
  int p = -1, c = -1, k = -1;
  if (mhc_fwd_workspace_size(16384, 4, 4096, &fw)) return 2;
  if (mhc_bwd_workspace_size_for(16384, 4, 4096, 148, &bw)) return 3;
  if (mhc_query_plan_for(1, 16384, 4, 4096, 148, &p, &c, &k)) return 4;
  printf("%d %zu %zu %d %d %d %s\n", mhc_abi_version(), fw, bw, p, c, k, mhc_status_string(MHC_ERR_LIMIT));
  return 0;
}
'''
    libdir = os.path.dirname(_lib.lib_path())
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "caller.c")
        exe = os.path.join(d, "caller")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-std=c99", "-I", os.path.join(ROOT, "include"), c, "-o", exe, "-L", libdir,
                        "-lmhc_ops", f"-Wl,-rpath,{libdir}"], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()
    lib = _lib.load()
    fw, bw = ctypes.c_size_t(0), ctypes.c_size_t(0)
    lib.mhc_fwd_workspace_size(16384, 4, 4096, ctypes.byref(fw))
    lib.mhc_bwd_workspace_size_for(16384, 4, 4096, 148, ctypes.byref(bw))
    plan = _lib.query_plan(1, 16384, 4, 4096, sms=148)
    assert int(out[0]) == lib.mhc_abi_version()
    assert (int(out[1]), int(out[2])) == (fw.value, bw.value)
    assert (int(out[3]), int(out[4]), int(out[5])) == (1, plan["d_slices"], plan["token_groups"])
    assert " ".join(out[6:]).encode() == lib.mhc_status_string(8)


def test_normal_build_has_no_bounds_checks(lib):
    """mhc_debug_bounds answers without a device in a normal build: unsupported, zero record."""
    rec = (ctypes.c_uint64 * 4)(1, 2, 3, 4)
    assert lib.mhc_debug_bounds(rec, 1) == _lib.MHC_ERR_UNSUPPORTED
    assert list(rec) == [0, 0, 0, 0]
    assert lib.mhc_debug_bounds(None, 0) == 1
    assert lib.mhc_debug_bounds_selftest(None, None) == _lib.MHC_ERR_UNSUPPORTED


def test_debug_bounds_build_exports_every_declared_symbol():
    """The -DMHC_DEBUG_BOUNDS library builds from the same sources and exports the same ABI."""
    from mhc_ops_b200 import build
    path = build.build(debug_bounds=True)
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (mhc_\w+)$", out, flags=re.M))
    assert not [s for s in _declared_symbols() if s not in exported]
