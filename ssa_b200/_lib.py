"""ctypes binding of the C ABI in include/ssa_b200.h (libssa_b200.so).

The library is loaded from the package directory. There is no fallback: if
the library is missing, or no CUDA device is present when a kernel is
called, the call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libssa_b200.so")

SSA_OK, SSA_ERR_INVALID, SSA_ERR_UNSUPPORTED, SSA_ERR_WORKSPACE, SSA_ERR_CUDA, SSA_ERR_DEVICE = range(6)
SSA_F32, SSA_BF16 = 0, 1
# Size of the static device scratch of ssa_attn_bwd_noalloc (the header's
# SSA_ATTN_BWD_STATIC_SCRATCH_BYTES).
SSA_ATTN_BWD_STATIC_SCRATCH_BYTES = 64 << 20

_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t


class GraphParams(ctypes.Structure):
    """ssa_graph_params."""
    _fields_ = [(n, _i32) for n in ("B", "H", "n_kv", "N", "M", "d", "dtype", "R", "max_p", "p_eff",
                                    "C", "T", "A", "causal", "is_cross", "K", "window", "G")] + \
               [(n, _i64) for n in ("q_sb", "q_sh", "q_sn", "k_sb", "k_sh", "k_sm")] + \
               [("q_row0", _i32), ("reserved0", _i32)]


class AttnParams(ctypes.Structure):
    """ssa_attn_params."""
    _fields_ = [(n, _i32) for n in ("B", "H", "n_kv", "N", "M", "d", "Kn", "dtype", "nb_i64",
                                    "fp32_weights")] + \
               [("scale", ctypes.c_float)] + \
               [(n, _i64) for n in ("q_sb", "q_sh", "q_sn", "k_sb", "k_sh", "k_sm",
                                    "v_sb", "v_sh", "v_sm", "o_sb", "o_sh", "o_sn")] + \
               [("dropout_p", ctypes.c_float), ("reserved0", _i32),
                ("dropout_seed", ctypes.c_uint64), ("dropout_offset", ctypes.c_uint64)]


# name -> (restype, argtypes): exactly the declarations of include/ssa_b200.h
SIGNATURES = {
    "ssa_graph_width": (_i32, [ctypes.POINTER(GraphParams)]),
    "ssa_graph_workspace_size": (_sz, [ctypes.POINTER(GraphParams)]),
    "ssa_build_graph": (ctypes.c_int, [ctypes.POINTER(GraphParams), _vp, _vp, _vp, _vp, _vp, _vp,
                                       _vp, _vp, _sz, _vp]),
    "ssa_lsh_select": (ctypes.c_int, [ctypes.POINTER(GraphParams), _vp, _vp, _vp, _vp, _vp, _vp,
                                      _sz, _vp]),
    "ssa_merge": (ctypes.c_int, [ctypes.POINTER(GraphParams), _vp, _vp, _vp, _i32, _vp, _vp, _vp,
                                 _vp, _vp]),
    "ssa_hash_ids": (ctypes.c_int, [_vp, _i32, _i32, _i32, _i32, _i32, _i64, _i64, _i64, _vp, _i32,
                                    _i32, _i32, _vp, _vp]),
    "ssa_attn_fwd": (ctypes.c_int, [ctypes.POINTER(AttnParams), _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                    _vp]),
    "ssa_attn_bwd_workspace_size": (_sz, [ctypes.POINTER(AttnParams)]),
    "ssa_attn_bwd": (ctypes.c_int, [ctypes.POINTER(AttnParams), _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                    _vp, _vp, _vp, _vp, _sz, _vp]),
    "ssa_attn_csr_size": (_sz, [ctypes.POINTER(AttnParams)]),
    "ssa_attn_build_csr": (ctypes.c_int, [ctypes.POINTER(AttnParams), _vp, _vp, _vp, _sz, _vp, _sz, _vp]),
    "ssa_attn_bwd_csr": (ctypes.c_int, [ctypes.POINTER(AttnParams), _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                        _vp, _vp, _vp, _vp, _sz, _vp, _sz, _vp]),
    "ssa_attn_bwd_noalloc": (ctypes.c_int, [ctypes.POINTER(AttnParams), _vp, _vp, _vp, _vp, _vp, _vp,
                                            _vp, _vp, _vp, _vp, _vp]),
    "ssa_neighbor_overlap": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _vp, _vp]),
    "ssa_device_error": (_i32, [_i32]),
    "ssa_debug_set_wait_limit": (ctypes.c_int, [ctypes.c_uint32]),
    "ssa_qkv_proj_hash_supported": (_i32, [ctypes.POINTER(GraphParams), _i32]),
    "ssa_qkv_proj_hash": (ctypes.c_int, [ctypes.POINTER(GraphParams), _i32, _vp, _vp, _vp, _vp, _vp, _sz,
                                         _vp]),
    "ssa_build_graph_prehashed": (ctypes.c_int, [ctypes.POINTER(GraphParams), _vp, _vp, _vp, _vp, _vp, _vp,
                                                 _vp, _sz, _vp]),
    "ssa_debug_set_hash": (ctypes.c_int, [_i32, ctypes.c_float]),
    "ssa_debug_hash_dump": (ctypes.c_int, [ctypes.c_void_p, _i64]),
    "ssa_debug_hash_recomputed": (_i64, [_i32]),
    "ssa_last_error": (ctypes.c_char_p, []),
    "ssa_abi_version": (_i32, []),
    "ssa_kernel_launches": (_i64, []),
    "ssa_graph_profile": (ctypes.c_int, [_i32]),
    "ssa_graph_stage_times": (ctypes.c_int, [ctypes.POINTER(ctypes.c_float)]),
}

# ssa_graph_stage_times order (the header's SSA_GRAPH_STAGES stages)
GRAPH_STAGES = ("hash_keys", "bucket_trim", "hash_queries", "scan_sample", "rows_thresh", "scan_full",
                "rows_final", "select_fma")

_lib = None
_lock = threading.Lock()


class SSAError(RuntimeError):
    pass


def load():
    """Load libssa_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise SSAError(f"{LIB_PATH} is missing: build it with `python -m ssa_b200.build`")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(rc: int, what: str):
    if rc == SSA_OK:
        return
    msg = load().ssa_last_error().decode(errors="replace")
    if rc in (SSA_ERR_INVALID, SSA_ERR_WORKSPACE):
        raise ValueError(f"{what}: {msg}")
    if rc == SSA_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise SSAError(f"{what} failed ({rc}): {msg}")
