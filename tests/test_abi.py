"""C-ABI checks that need no GPU: the library loads, exports every function
the headers under ``include/`` declare, and the ctypes mirror of every struct
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
HEADERS = [os.path.join(ROOT, "include", h)
           for h in ("bozo_tension.h", "bozo_tau_aux.h", "bozo_graph_bias.h", "bozo_block_ops.h")]


def _declared_functions():
    found = set()
    for h in HEADERS:
        src = open(h).read()
        found |= set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(bozo_\w+)\s*\(", src, re.M))
    return sorted(found)


def test_every_header_is_covered():
    assert sorted(os.listdir(os.path.join(ROOT, "include"))) == sorted(os.path.basename(h) for h in HEADERS)


def test_library_exports_every_declared_symbol():
    if not os.path.exists(_capi.LIB_PATH):
        pytest.skip("library not built")
    lib = _capi.lib()
    declared = _declared_functions()
    assert declared, "no declarations parsed"
    assert set(declared) == set(_capi.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.bozo_tension_abi_version() == 7
    assert _capi.status_string(0) == "ok"


PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "bozo_tension.h"
#include "bozo_tau_aux.h"
#include "bozo_graph_bias.h"
#include "bozo_block_ops.h"
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
  O(bozo_tension_fwd_args, k_rot); O(bozo_tension_fwd_args, q_lp); O(bozo_tension_fwd_args, k_lp); O(bozo_tension_bwd_args, qk_rotated);
  S(bozo_tension_bwd_args);
  O(bozo_tension_bwd_args, d_out); O(bozo_tension_bwd_args, out);
  O(bozo_tension_bwd_args, row_mass); O(bozo_tension_bwd_args, bias_stride);
  O(bozo_tension_bwd_args, d_tau); O(bozo_tension_bwd_args, grad_dtype);
  O(bozo_tension_bwd_args, dq); O(bozo_tension_bwd_args, workspace);
  O(bozo_tension_bwd_args, workspace_bytes); O(bozo_tension_bwd_args, aux_row);
  S(bozo_tension_decode_args); O(bozo_tension_decode_args, scale); O(bozo_tension_decode_args, pos);
  O(bozo_tension_decode_args, rope_len); O(bozo_tension_decode_args, rope_sin);
  O(bozo_tension_decode_args, q); O(bozo_tension_decode_args, v);
  O(bozo_tension_decode_args, k_cache); O(bozo_tension_decode_args, v_cache_dtype);
  O(bozo_tension_decode_args, out); O(bozo_tension_decode_args, tau);
  O(bozo_tension_decode_args, tau_dtype);
  S(bozo_add_rmsnorm_args); O(bozo_add_rmsnorm_args, eps); O(bozo_add_rmsnorm_args, y_dtype);
  O(bozo_add_rmsnorm_args, scale); O(bozo_add_rmsnorm_args, d_scale);
  O(bozo_add_rmsnorm_args, workspace_bytes); O(bozo_add_rmsnorm_args, out_lp);
  O(bozo_add_rmsnorm_args, d_out_lp);
  S(bozo_wo_add_rmsnorm_args); O(bozo_wo_add_rmsnorm_args, eps); O(bozo_wo_add_rmsnorm_args, msg);
  O(bozo_wo_add_rmsnorm_args, x_dtype); O(bozo_wo_add_rmsnorm_args, scale);
  O(bozo_wo_add_rmsnorm_args, rstd);
  S(bozo_swiglu_args); O(bozo_swiglu_args, gate); O(bozo_swiglu_args, d_value);
  O(bozo_swiglu_args, width); O(bozo_swiglu_args, row_stride);
  S(bozo_embedding_bwd_args); O(bozo_embedding_bwd_args, vocab); O(bozo_embedding_bwd_args, sorted_ids);
  O(bozo_embedding_bwd_args, d_weight); O(bozo_embedding_bwd_args, scratch);
  S(bozo_cross_entropy_args); O(bozo_cross_entropy_args, logits_dtype);
  O(bozo_cross_entropy_args, targets); O(bozo_cross_entropy_args, d_logits);
  S(bozo_graph_bias_args); O(bozo_graph_bias_args, alpha); O(bozo_graph_bias_args, ctx_content);
  O(bozo_graph_bias_args, n_edges); O(bozo_graph_bias_args, out); O(bozo_graph_bias_args, stats);
  S(bozo_tau_aux_fwd_args); O(bozo_tau_aux_fwd_args, W); O(bozo_tau_aux_fwd_args, tau);
  O(bozo_tau_aux_fwd_args, stats); O(bozo_tau_aux_fwd_args, workspace);
  O(bozo_tau_aux_fwd_args, workspace_bytes); O(bozo_tau_aux_fwd_args, row_ent);
  S(bozo_tau_aux_bwd_args); O(bozo_tau_aux_bwd_args, tau); O(bozo_tau_aux_bwd_args, d_stats);
  O(bozo_tau_aux_bwd_args, d_tau); O(bozo_tau_aux_bwd_args, row_coef);
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
             "bozo_tension_bwd_args": _capi.BwdArgs,
             "bozo_tension_decode_args": _capi.DecodeArgs,
             "bozo_graph_bias_args": _capi.GraphBiasArgs,
             "bozo_add_rmsnorm_args": _capi.AddRMSNormArgs,
             "bozo_swiglu_args": _capi.SwiGLUArgs,
             "bozo_wo_add_rmsnorm_args": _capi.WoAddRMSNormArgs,
             "bozo_cross_entropy_args": _capi.CrossEntropyArgs,
             "bozo_embedding_bwd_args": _capi.EmbeddingBwdArgs,
             "bozo_tau_aux_fwd_args": _capi.TauAuxFwdArgs,
             "bozo_tau_aux_bwd_args": _capi.TauAuxBwdArgs}
    for line in filter(None, lines):
        key, val = line.split()
        if "." in key:
            t, f = key.split(".")
            assert getattr(names[t], f).offset == int(val), key
        else:
            assert C.sizeof(names[key]) == int(val), key
