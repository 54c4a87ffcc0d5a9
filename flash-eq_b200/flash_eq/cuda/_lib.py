"""ctypes binding of libflasheq_b200.so (declarations: include/flasheq_b200.h).

The library is built in-tree by ``flash-eq_b200/csrc/Makefile`` into
``flash_eq/_lib/``.  There is no fallback: if the library is missing every op
raises ``ImportError`` with the build command.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "_lib", "libflasheq_b200.so")

FEQ_OK = 0
FEQ_BASIS_MFIRST = 0
FEQ_BASIS_ROT_TO_EZ = 1
FEQ_REDUCE = {"sum": 0, "mean": 1, "max": 2}
FEQ_MIX = {"fp32": 0, "bf16": 1, "bf16x3": 2}
MAX_L = 16

c_i32p = ctypes.POINTER(ctypes.c_int32)
c_vp = ctypes.c_void_p


class FeqEdgewiseArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_vp), ("src", c_vp), ("num_src_rows", ctypes.c_int64), ("edge_add", c_vp),
        ("directions", c_vp), ("P_in", c_vp), ("Q_out", c_vp), ("distances", c_vp),
        ("radial_table", c_vp), ("num_edges", ctypes.c_int64), ("c_in", ctypes.c_int32),
        ("c_out", ctypes.c_int32), ("lvals_in", c_i32p), ("n_lvals_in", ctypes.c_int32),
        ("lvals_out", c_i32p), ("n_lvals_out", ctypes.c_int32), ("sh_scale", ctypes.c_float),
        ("bin_param1", ctypes.c_float), ("bin_param2", ctypes.c_float), ("num_bins", ctypes.c_int32),
        ("log_bins", ctypes.c_int32), ("out", c_vp), ("status", c_vp), ("mix_mode", ctypes.c_int32),
    ]


class FeqSeparableArgs(ctypes.Structure):
    _fields_ = [
        ("x", c_vp), ("src", c_vp), ("num_src_rows", ctypes.c_int64), ("edge_add", c_vp),
        ("directions", c_vp), ("distances", c_vp), ("channel_patterns", c_vp), ("radial_features", c_vp),
        ("num_edges", ctypes.c_int64), ("c_in", ctypes.c_int32), ("c_out", ctypes.c_int32),
        ("rank", ctypes.c_int32), ("lvals_in", c_i32p), ("n_lvals_in", ctypes.c_int32),
        ("lvals_out", c_i32p), ("n_lvals_out", ctypes.c_int32), ("sh_scale", ctypes.c_float),
        ("bin_param1", ctypes.c_float), ("bin_param2", ctypes.c_float), ("num_bins", ctypes.c_int32),
        ("log_bins", ctypes.c_int32), ("out", c_vp), ("status", c_vp), ("mix_mode", ctypes.c_int32),
    ]


class FeqAttnArgs(ctypes.Structure):
    _fields_ = [
        ("qk", c_vp), ("v", c_vp), ("src", c_vp), ("distances", c_vp), ("perm", c_vp), ("offsets", c_vp),
        ("num_nodes", ctypes.c_int64), ("num_edges", ctypes.c_int64), ("c_qk", ctypes.c_int32),
        ("d_qk", ctypes.c_int32), ("c_v", ctypes.c_int32), ("d_v", ctypes.c_int32),
        ("num_heads", ctypes.c_int32), ("scale", ctypes.c_float), ("decay_scale", ctypes.c_float),
        ("reduce", ctypes.c_int32), ("out", c_vp), ("status", c_vp), ("k", c_vp),
        ("num_src_nodes", ctypes.c_int64),
    ]


class FeqAttnBwdArgs(ctypes.Structure):
    _fields_ = [
        ("fwd", FeqAttnArgs), ("grad_out", c_vp), ("dst", c_vp), ("src_perm", c_vp), ("src_offsets", c_vp),
        ("grad_q", c_vp), ("ldq", ctypes.c_int64), ("grad_k", c_vp), ("ldk", ctypes.c_int64), ("grad_v", c_vp),
        ("grad_distances", c_vp), ("grad_scale_partial", c_vp), ("edge_scratch", c_vp),
    ]


FEQ_ABI_VERSION = 4   # must equal feq_abi_version() of the loaded library

# name -> (restype, argtypes)
SIGNATURES = {
    "feq_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "feq_abi_version": (ctypes.c_int, []),
    "feq_last_error": (ctypes.c_char_p, []),
    "feq_launch_count": (ctypes.c_int64, []),
    "feq_set_wait_limit_ns": (ctypes.c_uint64, [ctypes.c_uint64]),
    "feq_profile_enable": (ctypes.c_int, [ctypes.c_int32]),
    "feq_profile_read": (ctypes.c_int, [ctypes.c_int32, ctypes.c_char_p, ctypes.c_int32,
                                        ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64)]),
    "feq_wigner_basis": (ctypes.c_int, [c_vp, ctypes.c_int64, c_i32p, ctypes.c_int32, ctypes.c_int32, c_vp, c_vp]),
    "feq_edge_binning": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_float, ctypes.c_float, ctypes.c_int32,
                                        ctypes.c_int32, c_vp, c_vp, c_vp]),
    "feq_edge_sort_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int32]),
    "feq_edge_sort": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, c_vp, c_vp, c_vp, c_vp,
                                     ctypes.c_size_t, c_vp]),
    "feq_edge_sort_i64": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, c_vp, c_vp, c_vp, c_vp,
                                         ctypes.c_size_t, c_vp]),
    "feq_block_diagonal_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                                             c_i32p, ctypes.c_int32, c_i32p, ctypes.c_int32,
                                                             ctypes.c_int32]),
    "feq_block_diagonal_fwd": (ctypes.c_int, [c_vp, c_vp, c_vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                              c_i32p, ctypes.c_int32, c_i32p, ctypes.c_int32, ctypes.c_float,
                                              ctypes.c_float, ctypes.c_float, ctypes.c_int32, ctypes.c_int32,
                                              c_vp, c_vp, ctypes.c_size_t, c_vp]),
    "feq_block_diagonal_fwd_mix_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int32,
                                                                     ctypes.c_int32, c_i32p, ctypes.c_int32, c_i32p,
                                                                     ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "feq_block_diagonal_fwd_mix": (ctypes.c_int, [c_vp, c_vp, c_vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                                  c_i32p, ctypes.c_int32, c_i32p, ctypes.c_int32, ctypes.c_float,
                                                  ctypes.c_float, ctypes.c_float, ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.c_int32, c_vp, c_vp, ctypes.c_size_t, c_vp]),
    "feq_block_diagonal_bwd_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                                                 c_i32p, ctypes.c_int32, c_i32p, ctypes.c_int32,
                                                                 ctypes.c_int32, ctypes.c_int32]),
    "feq_block_diagonal_bwd": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                              c_i32p, ctypes.c_int32, c_i32p, ctypes.c_int32, ctypes.c_float,
                                              ctypes.c_float, ctypes.c_float, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, c_vp, c_vp, c_vp, c_vp, ctypes.c_size_t, c_vp]),
    "feq_block_diagonal_fwd_noalloc": (ctypes.c_int, [c_vp, c_vp, c_vp, ctypes.c_int64, ctypes.c_int32,
                                                      ctypes.c_int32, c_i32p, ctypes.c_int32, c_i32p,
                                                      ctypes.c_int32, ctypes.c_float, ctypes.c_float,
                                                      ctypes.c_float, ctypes.c_int32, ctypes.c_int32, c_vp, c_vp]),
    "feq_edgewise_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(FeqEdgewiseArgs)]),
    "feq_edgewise_fwd": (ctypes.c_int, [ctypes.POINTER(FeqEdgewiseArgs), c_vp, ctypes.c_size_t, c_vp]),
    "feq_edgewise_separable_supported": (ctypes.c_int, [ctypes.POINTER(FeqSeparableArgs)]),
    "feq_edgewise_separable_fwd": (ctypes.c_int, [ctypes.POINTER(FeqSeparableArgs), c_vp]),
    "feq_segment_softmax": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, c_vp, c_vp, ctypes.c_int64,
                                           c_vp, c_vp]),
    "feq_edge_attention_weights": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.c_float, c_vp, ctypes.c_float, c_vp, c_vp,
                                                  ctypes.c_int64, c_vp, c_vp]),
    "feq_segment_pool": (ctypes.c_int, [c_vp, ctypes.c_int64, c_vp, ctypes.c_int32, c_vp, c_vp, ctypes.c_int64,
                                        ctypes.c_int32, c_vp, c_vp]),
    "feq_attn_pool_fwd": (ctypes.c_int, [ctypes.POINTER(FeqAttnArgs), c_vp]),
    "feq_attn_pool_bwd": (ctypes.c_int, [ctypes.POINTER(FeqAttnBwdArgs), c_vp]),
    "feq_node_sep_layernorm": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, c_i32p, ctypes.c_int32, c_vp,
                                              c_vp, c_vp, ctypes.c_float, c_vp, c_vp]),
    "feq_node_layernorm": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, c_i32p, ctypes.c_int32, c_vp, c_vp,
                                          ctypes.c_float, ctypes.c_float, ctypes.c_float, c_vp, c_vp]),
    "feq_node_rep_norm": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, c_i32p, ctypes.c_int32, ctypes.c_float,
                                         c_vp, c_vp]),
    "feq_node_to_posmajor": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, c_vp, c_vp]),
    "feq_dense_linear_tc_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "feq_dense_linear_tc": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, c_vp, c_vp,
                                           ctypes.c_int32, c_vp, c_vp, ctypes.c_size_t, c_vp, c_vp]),
    "feq_radial_features": (ctypes.c_int, [c_vp, ctypes.c_int32, ctypes.c_float, ctypes.c_float, c_vp, ctypes.c_int32,
                                           c_vp, c_vp, ctypes.c_int32, c_vp, c_vp, c_vp, c_vp, ctypes.c_int32, c_vp,
                                           c_vp]),
    "feq_node_linear_tc_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32, c_i32p, ctypes.c_int32,
                                                              ctypes.c_int32]),
    "feq_node_linear_tc": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, c_i32p, ctypes.c_int32,
                                          c_vp, c_vp, ctypes.c_int32, c_vp, c_vp, ctypes.c_size_t, c_vp, c_vp]),
    "feq_node_from_posmajor": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, c_i32p, ctypes.c_int32, c_vp,
                                              c_vp, c_vp, c_vp]),
    "feq_knn_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int64]),
    "feq_knn_graph": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_float,
                                     ctypes.c_float, ctypes.c_float, c_vp, c_vp, c_vp, ctypes.c_size_t, c_vp]),
    "feq_radius_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int64]),
    "feq_radius_pairs_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int64]),
    "feq_radius_count": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int64, ctypes.c_float, ctypes.c_int32, ctypes.c_float,
                                        ctypes.c_float, ctypes.c_float, ctypes.c_float, c_vp, c_vp, c_vp,
                                        ctypes.c_size_t, c_vp]),
    "feq_radius_fill": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int64, ctypes.c_float, ctypes.c_int32, ctypes.c_float,
                                       ctypes.c_float, ctypes.c_float, ctypes.c_float, c_vp, ctypes.c_int64, c_vp,
                                       c_vp, c_vp, ctypes.c_size_t, c_vp, ctypes.c_size_t, c_vp]),
    "feq_node_gate": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int64, ctypes.c_int32, c_i32p, ctypes.c_int32, c_vp, c_vp]),
    "feq_segment_softmax_bwd": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int64, ctypes.c_int32, c_vp, c_vp,
                                               ctypes.c_int64, c_vp, c_vp]),
    "feq_edge_attention_weights_bwd": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                                      ctypes.c_float, ctypes.c_float, c_vp, c_vp, ctypes.c_int64,
                                                      c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "feq_segment_pool_bwd": (ctypes.c_int, [c_vp, ctypes.c_int64, c_vp, ctypes.c_int32, c_vp, c_vp, c_vp,
                                            ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, c_vp, c_vp, c_vp, c_vp,
                                            c_vp, c_vp, c_vp]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the native library (no GPU needed to load it)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.isfile(LIB_PATH):
            raise ImportError(
                f"flash-eq B200 native library not found at {LIB_PATH}.\n"
                "Build it with:  make -C flash-eq_b200/csrc -j4   (or python -c 'import __graft_entry__ as g; g.build()')"
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.feq_abi_version() != FEQ_ABI_VERSION:
            raise ImportError(f"{LIB_PATH} has ABI version {lib.feq_abi_version()}, this package needs "
                              f"{FEQ_ABI_VERSION}: rebuild it with  make -C flash-eq_b200/csrc -j4")
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != FEQ_OK:
        lib = load()
        msg = lib.feq_status_string(rc).decode()
        extra = lib.feq_last_error().decode()
        raise RuntimeError(f"{what} failed: {msg}" + (f" ({extra})" if extra else ""))


def i32_array(vals):
    vals = [int(v) for v in vals]
    return (ctypes.c_int32 * max(1, len(vals)))(*vals), len(vals)
