"""ctypes binding of the C ABI declared in ``include/bozo_tension.h``,
``include/bozo_tau_aux.h``, ``include/bozo_graph_bias.h`` and
``include/bozo_block_ops.h``.

The structures below mirror the header field by field; ``tests/test_abi.py``
compiles a C probe with gcc and checks every size and offset, and checks
that the library exports every function the header declares.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib",
                        "libbozo_tension.so")

OK = 0
ERR_SCRATCH_LIMIT = 9
NOALLOC_SCRATCH_BYTES = 8 << 20  # BOZO_NOALLOC_SCRATCH_BYTES
DT_F32, DT_BF16, DT_F16 = 0, 1, 2
MODE_LOCAL, MODE_GLOBAL = 0, 1
NORM_NONE, NORM_MASS, NORM_COUNT = 0, 1, 2
PATH_AUTO, PATH_SIMT, PATH_TCGEN05 = 0, 1, 2

EXPORTED = (
    "bozo_tension_fwd", "bozo_tension_bwd", "bozo_tension_bwd_workspace",
    "bozo_tension_poll_error", "bozo_tension_last_path",
    "bozo_tension_last_launches", "bozo_status_string",
    "bozo_tension_abi_version", "bozo_tension_last_cuda_error",
    "bozo_tension_bwd_noalloc",
    "bozo_tau_aux_workspace", "bozo_tau_aux_fwd", "bozo_tau_aux_bwd",
    "bozo_tension_decode", "bozo_graph_bias_build",
    "bozo_add_rmsnorm_workspace", "bozo_add_rmsnorm_fwd", "bozo_add_rmsnorm_bwd",
    "bozo_swiglu_fwd", "bozo_swiglu_bwd",
    "bozo_cross_entropy_fwd", "bozo_cross_entropy_bwd",
    "bozo_tension_error_async", "bozo_tension_wait_selftest", "bozo_tension_fwd_needs_lp",
    "bozo_wo_add_rmsnorm_fwd", "bozo_wo_add_rmsnorm_supported",
    "bozo_embedding_bwd",
)
TAU_AUX_MAX_LAYERS = 64  # BOZO_TAU_AUX_MAX_LAYERS


class Tensor4(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("dtype", C.c_int32), ("_pad", C.c_int32),
                ("stride", C.c_int64 * 4)]


class FwdArgs(C.Structure):
    _fields_ = [
        ("B", C.c_int32), ("T", C.c_int32), ("H", C.c_int32), ("HD", C.c_int32),
        ("mode", C.c_int32), ("window", C.c_int32), ("normalize", C.c_int32),
        ("path", C.c_int32), ("scale", C.c_float), ("rope_len", C.c_int32),
        ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p), ("rope_theta", C.c_void_p),
        ("q", Tensor4), ("k", Tensor4), ("v", Tensor4),
        ("bias", C.c_void_p), ("bias_stride", C.c_int64 * 3),
        ("out", C.c_void_p), ("out_dtype", C.c_int32), ("tau_dtype", C.c_int32),
        ("tau", C.c_void_p), ("row_mass", C.c_void_p),
        ("q_rot", C.c_void_p), ("k_rot", C.c_void_p),
        ("q_lp", C.c_void_p), ("k_lp", C.c_void_p),
    ]


class BwdArgs(C.Structure):
    _fields_ = [
        ("B", C.c_int32), ("T", C.c_int32), ("H", C.c_int32), ("HD", C.c_int32),
        ("mode", C.c_int32), ("window", C.c_int32), ("normalize", C.c_int32),
        ("path", C.c_int32), ("scale", C.c_float), ("rope_len", C.c_int32),
        ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p), ("rope_theta", C.c_void_p),
        ("q", Tensor4), ("k", Tensor4), ("v", Tensor4), ("d_out", Tensor4),
        ("out", Tensor4), ("row_mass", C.c_void_p),
        ("bias", C.c_void_p), ("bias_stride", C.c_int64 * 3),
        ("d_tau", C.c_void_p), ("d_tau_dtype", C.c_int32),
        ("grad_dtype", C.c_int32 * 3), ("qk_rotated", C.c_int32),
        ("dq", C.c_void_p), ("dk", C.c_void_p), ("dv", C.c_void_p),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("aux_row", C.c_void_p),
    ]


class DecodeArgs(C.Structure):
    _fields_ = [
        ("B", C.c_int32), ("H", C.c_int32), ("HD", C.c_int32), ("mode", C.c_int32),
        ("window", C.c_int32), ("normalize", C.c_int32), ("capacity", C.c_int32),
        ("tau_width", C.c_int32), ("scale", C.c_float), ("pos", C.c_void_p),
        ("rope_len", C.c_int32), ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p),
        ("q", Tensor4), ("k", Tensor4), ("v", Tensor4),
        ("k_cache", C.c_void_p), ("k_cache_dtype", C.c_int32),
        ("v_cache", C.c_void_p), ("v_cache_dtype", C.c_int32),
        ("out", C.c_void_p), ("out_dtype", C.c_int32),
        ("tau", C.c_void_p), ("tau_dtype", C.c_int32),
    ]


class AddRMSNormArgs(C.Structure):
    _fields_ = [
        ("rows", C.c_int64), ("width", C.c_int32), ("eps", C.c_float),
        ("x", C.c_void_p), ("x_dtype", C.c_int32), ("y", C.c_void_p), ("y_dtype", C.c_int32),
        ("scale", C.c_void_p), ("out", C.c_void_p), ("rstd", C.c_void_p),
        ("d_out", C.c_void_p), ("dx", C.c_void_p), ("dy", C.c_void_p), ("d_scale", C.c_void_p),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("out_lp", C.c_void_p), ("d_out_lp", C.c_void_p),
    ]


class WoAddRMSNormArgs(C.Structure):
    _fields_ = [
        ("rows", C.c_int64), ("width", C.c_int32), ("eps", C.c_float),
        ("msg", C.c_void_p), ("wo", C.c_void_p), ("x", C.c_void_p), ("x_dtype", C.c_int32),
        ("scale", C.c_void_p), ("out", C.c_void_p), ("rstd", C.c_void_p),
    ]


class SwiGLUArgs(C.Structure):
    _fields_ = [
        ("n", C.c_int64), ("dtype", C.c_int32), ("gate", C.c_void_p), ("value", C.c_void_p),
        ("out", C.c_void_p), ("d_out", C.c_void_p), ("d_gate", C.c_void_p), ("d_value", C.c_void_p),
        ("width", C.c_int64), ("row_stride", C.c_int64),
    ]


class EmbeddingBwdArgs(C.Structure):
    _fields_ = [
        ("n", C.c_int64), ("dim", C.c_int32), ("vocab", C.c_int32), ("sorted_ids", C.c_void_p),
        ("order", C.c_void_p), ("d_out", C.c_void_p), ("d_weight", C.c_void_p),
        ("scratch", C.c_void_p),
    ]


class CrossEntropyArgs(C.Structure):
    _fields_ = [
        ("rows", C.c_int64), ("vocab", C.c_int32), ("logits", C.c_void_p),
        ("logits_dtype", C.c_int32), ("targets", C.c_void_p), ("row_lse", C.c_void_p),
        ("row_loss", C.c_void_p), ("d_scale", C.c_void_p), ("d_logits", C.c_void_p),
    ]


class GraphBiasArgs(C.Structure):
    _fields_ = [
        ("T", C.c_int32), ("window", C.c_int32), ("alpha", C.c_double),
        ("ctx_content", C.c_void_p), ("edge_keys", C.c_void_p), ("edge_weights", C.c_void_p),
        ("n_edges", C.c_int64), ("out", C.c_void_p), ("stats", C.c_void_p),
    ]


class TauAuxFwdArgs(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int32), ("dtype", C.c_int32),
        ("B", C.c_int32), ("T", C.c_int32), ("H", C.c_int32), ("W", C.c_int32),
        ("tau", C.c_void_p * TAU_AUX_MAX_LAYERS), ("stats", C.c_void_p),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("row_ent", C.c_void_p),
    ]


class TauAuxBwdArgs(C.Structure):
    _fields_ = [
        ("n_layers", C.c_int32), ("dtype", C.c_int32),
        ("B", C.c_int32), ("T", C.c_int32), ("H", C.c_int32), ("W", C.c_int32),
        ("tau", C.c_void_p * TAU_AUX_MAX_LAYERS), ("d_stats", C.c_void_p),
        ("d_tau", C.c_void_p * TAU_AUX_MAX_LAYERS),
        ("row_coef", C.c_void_p * TAU_AUX_MAX_LAYERS),
    ]


_lib = None
_ext = None
_lock = threading.Lock()


def lib():
    """Load the in-tree shared library (raises if it was never built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with `python -m bozo_b200.build` "
                        "(the operator has no CPU fallback)")
                L = C.CDLL(LIB_PATH)
                L.bozo_tension_fwd.argtypes = [C.POINTER(FwdArgs), C.c_void_p]
                L.bozo_tension_fwd.restype = C.c_int
                L.bozo_tension_fwd_needs_lp.argtypes = [C.POINTER(FwdArgs)]
                L.bozo_tension_fwd_needs_lp.restype = C.c_int
                L.bozo_tension_bwd.argtypes = [C.POINTER(BwdArgs), C.c_void_p]
                L.bozo_tension_bwd.restype = C.c_int
                L.bozo_tension_bwd_noalloc.argtypes = [C.POINTER(BwdArgs), C.c_void_p]
                L.bozo_tension_bwd_noalloc.restype = C.c_int
                L.bozo_tension_bwd_workspace.argtypes = [C.POINTER(BwdArgs)]
                L.bozo_tension_bwd_workspace.restype = C.c_size_t
                L.bozo_tension_poll_error.argtypes = [C.c_void_p]
                L.bozo_tension_poll_error.restype = C.c_int
                L.bozo_tension_error_async.argtypes = [C.c_void_p, C.c_void_p]
                L.bozo_tension_error_async.restype = C.c_int
                L.bozo_tension_wait_selftest.argtypes = [C.c_uint64, C.c_void_p, C.c_void_p]
                L.bozo_tension_wait_selftest.restype = C.c_int
                L.bozo_tension_last_path.restype = C.c_int
                L.bozo_tension_last_launches.restype = C.c_int
                L.bozo_status_string.argtypes = [C.c_int]
                L.bozo_status_string.restype = C.c_char_p
                L.bozo_tension_abi_version.restype = C.c_int
                L.bozo_tension_last_cuda_error.restype = C.c_char_p
                L.bozo_graph_bias_build.argtypes = [C.POINTER(GraphBiasArgs), C.c_void_p]
                L.bozo_graph_bias_build.restype = C.c_int
                L.bozo_tension_decode.argtypes = [C.POINTER(DecodeArgs), C.c_void_p]
                L.bozo_tension_decode.restype = C.c_int
                L.bozo_tau_aux_workspace.argtypes = [C.POINTER(TauAuxFwdArgs)]
                L.bozo_tau_aux_workspace.restype = C.c_size_t
                L.bozo_tau_aux_fwd.argtypes = [C.POINTER(TauAuxFwdArgs), C.c_void_p]
                L.bozo_tau_aux_fwd.restype = C.c_int
                L.bozo_tau_aux_bwd.argtypes = [C.POINTER(TauAuxBwdArgs), C.c_void_p]
                L.bozo_tau_aux_bwd.restype = C.c_int
                L.bozo_wo_add_rmsnorm_fwd.argtypes = [C.POINTER(WoAddRMSNormArgs), C.c_void_p]
                L.bozo_wo_add_rmsnorm_fwd.restype = C.c_int
                L.bozo_wo_add_rmsnorm_supported.argtypes = [C.c_int32, C.c_int32]
                L.bozo_wo_add_rmsnorm_supported.restype = C.c_int
                _lib = L
    return _lib


def ext():
    """The PyTorch C++ extension (``_torch_ext``) that calls the C ABI for the
    autograd functions; built beside the library by ``bozo_b200.build``."""
    global _ext
    if _ext is None:
        lib()  # the extension links against the library: fail with its message first
        with _lock:
            if _ext is None:
                import glob
                import importlib.util
                found = glob.glob(os.path.join(os.path.dirname(LIB_PATH), "_torch_ext*.so"))
                if not found:
                    raise ImportError("the bozo_b200 torch extension is missing: build it with "
                                      "`python -m bozo_b200.build`")
                spec = importlib.util.spec_from_file_location("_torch_ext", found[0])
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                _ext = mod
    return _ext


def status_string(code: int) -> str:
    return lib().bozo_status_string(code).decode()


def check(code: int, what: str):
    if code != OK:
        detail = ""
        if code == 7:  # BOZO_ERR_CUDA
            detail = f" [{lib().bozo_tension_last_cuda_error().decode()}]"
        raise RuntimeError(f"{what} failed: {status_string(code)} (status {code}){detail}")
