"""numpy front end of the C oracle (ssa_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by `__graft_entry__.smoke()` as
the checker, and by bench.py's CPU-baseline leg. The ssa_b200 package never
imports it.

`build()` compiles ssa_oracle.c with gcc/OpenMP into oracle/_build/. The
functions below take numpy arrays in the layouts documented in ssa_oracle.c
and mirror the reference's hot-path entry points:

    lsh_select  -> LSHGraphBuilder.forward       (sparse_attention.py:814-959)
    merge       -> WindowGraphBuilder + merge_neighbors (:357-376, :966-1089)
    build_graph -> SparseAttention.build_graph    (:1325-1390)
    attn_fwd    -> sparse_gather_attention        (:1096-1199)
    attn_bwd    -> its autograd backward
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from typing import List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(BUILD_DIR, "libssa_oracle.so")
SRC = os.path.join(HERE, "ssa_oracle.c")

_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle shared library (gcc, -O2, OpenMP)."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(SRC):
        tmp = LIB_PATH + f".tmp{os.getpid()}"
        subprocess.check_call(["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-Wall",
                               "-o", tmp, SRC, "-lm"])
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        I = ctypes.c_int
        L.ora_effective_p.argtypes = [ctypes.c_int64, ctypes.c_int64, I]
        L.ora_lsh_select.argtypes = [P, P, I, I, I, I, I, I, P, I, I, I, I, I, I, I,
                                     P, I, P, P, P]
        L.ora_merge_width.argtypes = [I, I, I]
        L.ora_merge.argtypes = [P, I, I, I, I, I, I, P, I, I, I, I, P, P]
        L.ora_attn_fwd.argtypes = [P, P, P, P, P, I, I, I, I, I, I, I, ctypes.c_float,
                                   I, I, P, P]
        L.ora_attn_bwd.argtypes = [P, P, P, P, P, P, I, I, I, I, I, I, I, ctypes.c_float,
                                   I, I, P, P, P]
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def num_threads() -> int:
    return int(lib().ora_num_threads())


def derived(K: int, w: int, n_glob: int, R: int, maxP: int, T: int, M: int):
    """lsh_k, C, p_eff, T_eff, A as the reference derives them
    (sparse_attention.py:1262-1266, :1294, :552-557, :629, :898)."""
    guaranteed = 2 * w + 1 + n_glob + 1
    lsh_k = max(K - guaranteed, 8)
    C = 4 * lsh_k
    p = int(lib().ora_effective_p(M, C, maxP))
    Te = min(T, p)
    A = min(lsh_k, R * C * (1 + Te))
    return dict(lsh_k=lsh_k, C=C, p_eff=p, T_eff=Te, A=A)


def lsh_select(q, k, rand_proj, *, n_kv: int, R: int, maxP: int, p: int, C: int,
               T: int, A: int, causal: bool, glob: Sequence[int], want_ids=False):
    q = _f32(q)
    k = _f32(k)
    B, H, N, d = q.shape
    M = k.shape[2]
    rp = _f32(rand_proj)
    g = _i32(np.asarray(list(glob), dtype=np.int32).reshape(-1))
    out = np.empty((B, H, N, A), dtype=np.int32)
    kid = np.empty((B * H, R, M), dtype=np.int32) if want_ids else None
    qid = np.empty((B * H, R, N), dtype=np.int32) if want_ids else None
    rc = lib().ora_lsh_select(_ptr(q), _ptr(k), B, H, n_kv, N, M, d, _ptr(rp), R, maxP,
                              p, C, T, A, int(causal), _ptr(g), g.size, _ptr(out),
                              _ptr(kid), _ptr(qid))
    if rc:
        raise RuntimeError(f"ora_lsh_select failed ({rc})")
    return (out, kid, qid) if want_ids else out


def merge(lsh, *, M: int, w: int, glob: Sequence[int], causal: bool, is_cross: bool, K: int):
    lsh = _i32(lsh)
    B, H, N, A = lsh.shape
    g = _i32(np.asarray(list(glob), dtype=np.int32).reshape(-1))
    Kw = 0 if is_cross else 2 * w + 1
    Kout = int(lib().ora_merge_width(K, Kw + g.size + A, int(is_cross)))
    nb = np.empty((B, H, N, Kout), dtype=np.int32)
    valid = np.empty((B, H, N, Kout), dtype=np.uint8)
    rc = lib().ora_merge(_ptr(lsh), B, H, N, M, A, w, _ptr(g), g.size, int(causal),
                         int(is_cross), K, _ptr(nb), _ptr(valid))
    if rc:
        raise RuntimeError(f"ora_merge failed ({rc})")
    return nb, valid.astype(bool)


def glob_list(M: int, G: int, explicit: Optional[List[int]]):
    """GlobalGraphBuilder.forward (sparse_attention.py:411-415)."""
    if explicit is not None:
        return [min(max(int(x), 0), M - 1) for x in explicit]
    return list(range(min(G, M)))


def build_graph(q, k, rand_proj, *, n_kv, K, w, G, glob_idx, R, maxP, T, causal,
                is_cross):
    """SparseAttention.build_graph (sparse_attention.py:1325-1390) on numpy
    inputs: q (B,H,N,d), k (B,n_kv,M,d)."""
    M = k.shape[2]
    glob = glob_list(M, G, glob_idx)
    n_glob = len(glob_idx) if glob_idx is not None else G
    dv = derived(K, w, n_glob, R, maxP, T, M)
    causal = bool(causal) and not is_cross
    lsh = lsh_select(q, k, rand_proj, n_kv=n_kv, R=R, maxP=maxP, p=dv["p_eff"], C=dv["C"],
                     T=T, A=dv["A"], causal=causal, glob=glob)
    return merge(lsh, M=M, w=w, glob=glob, causal=causal, is_cross=is_cross, K=K)


def attn_fwd(q, k, v, nb, valid, *, scale: float, lowp: bool, fp32_w: bool):
    q, k, v = _f32(q), _f32(k), _f32(v)
    nb = _i32(nb)
    vm = np.ascontiguousarray(valid, dtype=np.uint8)
    B, H, N, d = q.shape
    n_kv, M = k.shape[1], k.shape[2]
    Kn = nb.shape[-1]
    out = np.empty_like(q)
    lse = np.empty((B, H, N), dtype=np.float32)
    rc = lib().ora_attn_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(nb), _ptr(vm), B, H, n_kv, N, M,
                            d, Kn, float(scale), int(lowp), int(fp32_w), _ptr(out), _ptr(lse))
    if rc:
        raise RuntimeError(f"ora_attn_fwd failed ({rc})")
    return out, lse


def attn_bwd(q, k, v, nb, valid, dO, *, scale: float, lowp: bool, fp32_w: bool):
    q, k, v, dO = _f32(q), _f32(k), _f32(v), _f32(dO)
    nb = _i32(nb)
    vm = np.ascontiguousarray(valid, dtype=np.uint8)
    B, H, N, d = q.shape
    n_kv, M = k.shape[1], k.shape[2]
    Kn = nb.shape[-1]
    dq = np.empty_like(q)
    dk = np.empty_like(k)
    dv = np.empty_like(v)
    rc = lib().ora_attn_bwd(_ptr(q), _ptr(k), _ptr(v), _ptr(nb), _ptr(vm), _ptr(dO), B, H, n_kv,
                            N, M, d, Kn, float(scale), int(lowp), int(fp32_w), _ptr(dq),
                            _ptr(dk), _ptr(dv))
    if rc:
        raise RuntimeError(f"ora_attn_bwd failed ({rc})")
    return dq, dk, dv


def hash_proj(x, planes):
    """Hyperplane projections in float64 (the oracle's hash arithmetic), used
    to attribute hash disagreements to near-zero projections."""
    return np.asarray(x, dtype=np.float64) @ np.asarray(planes, dtype=np.float64).T
