"""C-ABI checks that need no GPU: the library loads, exports every function
``include/bozo_tension.h`` declares, and the ctypes mirror of every struct
matches the C layout (sizes and offsets measured by a gcc-compiled probe)."""
import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

from bozo_b200 import _capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bozo_tension.h")


def _declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(bozo_\w+)\s*\(", src, re.M)))


def test_library_exports_every_declared_symbol():
    if not os.path.exists(_capi.LIB_PATH):
        pytest.skip("library not built")
    lib = _capi.lib()
    declared = _declared_functions()
    assert declared, "no declarations parsed"
    assert set(declared) == set(_capi.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.bozo_tension_abi_version() == 3
    assert _capi.status_string(0) == "ok"


PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "bozo_tension.h"
#define O(T, f) printf(#T "." #f " %zu\n", offsetof(T, f))
#define S(T) printf(#T " %zu\n", sizeof(T))
int main(void) {
  S(bozo_tensor4); O(bozo_tensor4, dtype); O(bozo_tensor4, stride);
  S(bozo_tension_fwd_args);
  O(bozo_tension_fwd_args, scale); O(bozo_tension_fwd_args, rope_cos);
  O(bozo_tension_fwd_args, rope_theta); O(bozo_tension_bwd_args, rope_theta);
  O(bozo_tension_fwd_args, q); O(bozo_tension_fwd_args, v); O(bozo_tension_fwd_args, bias);
  O(bozo_tension_fwd_args, bias_stride); O(bozo_tension_fwd_args, out);
  O(bozo_tension_fwd_args, out_dtype); O(bozo_tension_fwd_args, tau);
  O(bozo_tension_fwd_args, row_mass); O(bozo_tension_fwd_args, q_rot);
  O(bozo_tension_fwd_args, k_rot); O(bozo_tension_bwd_args, qk_rotated);
  S(bozo_tension_bwd_args);
  O(bozo_tension_bwd_args, d_out); O(bozo_tension_bwd_args, out);
  O(bozo_tension_bwd_args, row_mass); O(bozo_tension_bwd_args, bias_stride);
  O(bozo_tension_bwd_args, d_tau); O(bozo_tension_bwd_args, grad_dtype);
  O(bozo_tension_bwd_args, dq); O(bozo_tension_bwd_args, workspace);
  O(bozo_tension_bwd_args, workspace_bytes);
  return 0;
}
"""


def test_struct_layout_matches_header():
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(c, "w").write(PROBE)
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        lines = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split("\n")
    names = {"bozo_tensor4": _capi.Tensor4, "bozo_tension_fwd_args": _capi.FwdArgs,
             "bozo_tension_bwd_args": _capi.BwdArgs}
    for line in filter(None, lines):
        key, val = line.split()
        if "." in key:
            t, f = key.split(".")
            assert getattr(names[t], f).offset == int(val), key
        else:
            assert C.sizeof(names[key]) == int(val), key
