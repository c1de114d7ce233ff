"""Torch-facing wrappers of the C ABI: tensors in, tensors out.

Every function here launches sm_100a kernels from libssa_b200.so on the
current CUDA stream. Tensors must live on a CUDA device; there is no CPU
path. Query-side tensors are (B, H, N, d) and key/value tensors
(B, n_kv, M, d), each with any strides whose last axis is contiguous -- so
the (B, N, H*d) outputs of the q/k/v projections are consumed without a
transpose or a GQA repeat.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import AttnParams, GraphParams, SSA_BF16, SSA_F32, check


def _require_cuda(*ts: torch.Tensor):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("ssa_b200 runs on CUDA tensors only (there is no CPU path); "
                               f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return SSA_F32
    if t.dtype == torch.bfloat16:
        return SSA_BF16
    raise NotImplementedError(f"ssa_b200 kernels take float32 or bfloat16 tensors, got {t.dtype}")


def _rows(t: torch.Tensor) -> Tuple[torch.Tensor, int, int, int]:
    """A 4-D tensor with a contiguous last axis and 4-element-aligned strides
    (copying only if needed), plus its first three strides."""
    if t.dim() != 4:
        raise ValueError(f"expected a 4-D tensor, got shape {tuple(t.shape)}")
    s = t.stride()
    es = t.element_size()
    ok = (s[3] == 1 and all(x % 4 == 0 for x in s[:3]) and
          t.data_ptr() % (16 if es == 4 else 8) == 0)
    if not ok:
        t = t.contiguous()
        s = t.stride()
    return t, s[0], s[1], s[2]


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def graph_params(q, k, *, R, max_p, p_eff, C, T, A, causal, is_cross, K, window, G, q_row0=0):
    B, H, N, d = q.shape
    Bk, n_kv, M, dk = k.shape
    if Bk != B or dk != d:
        raise ValueError(f"q {tuple(q.shape)} and k {tuple(k.shape)} disagree")
    if H % n_kv:
        raise ValueError(f"num_heads ({H}) must be divisible by num_kv_heads ({n_kv})")
    p = GraphParams()
    p.B, p.H, p.n_kv, p.N, p.M, p.d = B, H, n_kv, N, M, d
    p.dtype = _dtype_code(q)
    p.R, p.max_p, p.p_eff, p.C, p.T, p.A = R, max_p, p_eff, C, T, A
    p.causal, p.is_cross, p.K, p.window, p.G = int(causal), int(is_cross), K, window, G
    p.q_row0 = int(q_row0)
    return p


def _graph_inputs(q, k, rand_proj, glob):
    _require_cuda(q, k, rand_proj, glob)
    if q.dtype != k.dtype:
        raise ValueError(f"q and k dtypes differ ({q.dtype} vs {k.dtype})")
    q, qsb, qsh, qsn = _rows(q)
    k, ksb, ksh, ksm = _rows(k)
    rp = rand_proj.detach().to(torch.float32).contiguous()
    g = glob.to(torch.int32).contiguous() if glob is not None else None
    return q, (qsb, qsh, qsn), k, (ksb, ksh, ksm), rp, g


class PrehashedGraph:
    """The graph-build state a fused QKV projection leaves behind
    (ssa_qkv_proj_hash): its params, the workspace holding the hash state,
    the hyperplanes and the global indices, for build_graph_prehashed."""

    def __init__(self, params, ws, rand_proj, glob):
        self.params, self.ws, self.rand_proj, self.glob = params, ws, rand_proj, glob


def qkv_project_hash(x: torch.Tensor, w_qkv: torch.Tensor, rand_proj: torch.Tensor, glob: torch.Tensor, *,
                     H: int, n_kv: int, R: int, max_p: int, p_eff: int, C: int, T: int, A: int,
                     causal: bool, K: int, window: int):
    """Fused QKV projection + LSH hash (ssa_qkv_proj_hash): qkv = x w_qkv^T
    as (B, N, (H + 2 n_kv) d) bf16 with w_qkv = [Wq; Wk; Wv], and the hash
    state of the self-attention graph over its q / k views. Returns
    (qkv, PrehashedGraph), or None when the fused path does not serve these
    shapes (ssa_qkv_proj_hash_supported)."""
    _require_cuda(x, w_qkv, rand_proj, glob)
    if x.dim() != 3 or w_qkv.dim() != 2 or x.dtype != torch.bfloat16 or w_qkv.dtype != torch.bfloat16:
        return None
    B, N, dm = x.shape
    n_out = w_qkv.shape[0]
    if w_qkv.shape[1] != dm or n_out % (H + 2 * n_kv):
        raise ValueError(f"w_qkv {tuple(w_qkv.shape)} does not match x {tuple(x.shape)} and the heads")
    d = n_out // (H + 2 * n_kv)
    x = x.contiguous()
    w = w_qkv.contiguous()
    qkv = torch.empty((B, N, n_out), dtype=torch.bfloat16, device=x.device)
    q, k, _ = split_qkv(qkv, H, n_kv)
    rp = rand_proj.detach().to(torch.float32).contiguous()
    g = glob.to(torch.int32).contiguous() if glob is not None else None
    p = graph_params(q, k, R=R, max_p=max_p, p_eff=p_eff, C=C, T=T, A=A, causal=causal, is_cross=False,
                     K=K, window=window, G=g.numel() if g is not None else 0)
    p.q_sb, p.q_sh, p.q_sn = q.stride()[:3]
    p.k_sb, p.k_sh, p.k_sm = k.stride()[:3]
    L = _lib.load()
    if not L.ssa_qkv_proj_hash_supported(ctypes.byref(p), dm):
        return None
    ws_bytes = L.ssa_graph_workspace_size(ctypes.byref(p))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    check(L.ssa_qkv_proj_hash(ctypes.byref(p), dm, _ptr(x), _ptr(w), _ptr(qkv), _ptr(rp), _ptr(ws), ws_bytes,
                              _stream(x.device)), "ssa_qkv_proj_hash")
    return qkv, PrehashedGraph(p, ws, rp, g)


def split_qkv(qkv: torch.Tensor, H: int, n_kv: int):
    """(B, N, (H + 2 n_kv) d) -> q (B, H, N, d), k, v (B, n_kv, N, d) views."""
    B, N, n_out = qkv.shape
    d = n_out // (H + 2 * n_kv)
    q = qkv[..., :H * d].view(B, N, H, d).transpose(1, 2)
    k = qkv[..., H * d:(H + n_kv) * d].view(B, N, n_kv, d).transpose(1, 2)
    v = qkv[..., (H + n_kv) * d:].view(B, N, n_kv, d).transpose(1, 2)
    return q, k, v


def build_graph_prehashed(q: torch.Tensor, k: torch.Tensor, state: PrehashedGraph):
    """ssa_build_graph_prehashed: the graph of the q / k views of a fused
    projection's output, from the hash state it left; the same result as
    build_graph on those views. Returns int32 neighbors and uint8 valid."""
    p, ws = state.params, state.ws
    L = _lib.load()
    W = L.ssa_graph_width(ctypes.byref(p))
    B, H, N = q.shape[:3]
    nb = torch.empty((B, H, N, W), dtype=torch.int32, device=q.device)
    valid = torch.empty((B, H, N, W), dtype=torch.uint8, device=q.device)
    check(L.ssa_build_graph_prehashed(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(state.rand_proj), _ptr(state.glob),
                                      _ptr(nb), _ptr(valid), _ptr(ws), ws.numel(), _stream(q.device)),
          "ssa_build_graph_prehashed")
    return nb, valid


def build_graph(q: torch.Tensor, k: torch.Tensor, rand_proj: torch.Tensor, glob: torch.Tensor, *,
                R: int, max_p: int, p_eff: int, C: int, T: int, A: int, causal: bool,
                is_cross: bool, K: int, window: int, want_lsh: bool = False, q_row0: int = 0):
    """SparseAttention.build_graph on the GPU. Returns int32 neighbors
    (B,H,N,W), uint8 valid (B,H,N,W) and, if asked, the int32 LSH set.
    q_row0: sequence position of q's first row when q holds a slice of the
    query rows (query-row sharding); k always holds every key."""
    q, qs, k, ks, rp, g = _graph_inputs(q, k, rand_proj, glob)
    G = g.numel() if g is not None else 0
    p = graph_params(q, k, R=R, max_p=max_p, p_eff=p_eff, C=C, T=T, A=A, causal=causal,
                     is_cross=is_cross, K=K, window=window, G=G, q_row0=q_row0)
    p.q_sb, p.q_sh, p.q_sn = qs
    p.k_sb, p.k_sh, p.k_sm = ks
    L = _lib.load()
    W = L.ssa_graph_width(ctypes.byref(p))
    ws_bytes = L.ssa_graph_workspace_size(ctypes.byref(p))
    if ws_bytes == 0:
        check(L.ssa_build_graph(ctypes.byref(p), None, None, None, None, None, None, None, None, 0,
                                None), "ssa_build_graph")
    B, H, N = q.shape[:3]
    dev = q.device
    nb = torch.empty((B, H, N, W), dtype=torch.int32, device=dev)
    valid = torch.empty((B, H, N, W), dtype=torch.uint8, device=dev)
    lsh = torch.empty((B, H, N, A), dtype=torch.int32, device=dev) if want_lsh else None
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    check(L.ssa_build_graph(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(rp), _ptr(g), _ptr(nb),
                            _ptr(valid), _ptr(lsh), _ptr(ws), ws_bytes, _stream(dev)),
          "ssa_build_graph")
    return (nb, valid, lsh) if want_lsh else (nb, valid)


def lsh_select(q, k, rand_proj, glob, *, R, max_p, p_eff, C, T, A, causal):
    """LSHGraphBuilder.forward on the GPU: (B,H,N,A) int32, reference order."""
    q, qs, k, ks, rp, g = _graph_inputs(q, k, rand_proj, glob)
    G = g.numel() if g is not None else 0
    p = graph_params(q, k, R=R, max_p=max_p, p_eff=p_eff, C=C, T=T, A=A, causal=causal,
                     is_cross=False, K=1, window=0, G=G)
    p.q_sb, p.q_sh, p.q_sn = qs
    p.k_sb, p.k_sh, p.k_sm = ks
    L = _lib.load()
    ws_bytes = L.ssa_graph_workspace_size(ctypes.byref(p))
    if ws_bytes == 0:
        check(L.ssa_lsh_select(ctypes.byref(p), None, None, None, None, None, None, 0, None),
              "ssa_lsh_select")
    B, H, N = q.shape[:3]
    dev = q.device
    out = torch.empty((B, H, N, A), dtype=torch.int32, device=dev)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    check(L.ssa_lsh_select(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(rp), _ptr(g), _ptr(out),
                           _ptr(ws), ws_bytes, _stream(dev)), "ssa_lsh_select")
    return out


def merge(win: torch.Tensor, glob: torch.Tensor, lsh: torch.Tensor, self_idx: Optional[torch.Tensor],
          total_k: int):
    """merge_neighbors on the GPU for explicit window/global/LSH/self
    tensors. Returns int32 neighbors and uint8 valid."""
    _require_cuda(win, glob, lsh, self_idx)
    B, H, N, A = lsh.shape
    win32 = win.to(torch.int32).reshape(N, -1).contiguous()
    Kw = win32.shape[1]
    g = glob.to(torch.int32).reshape(-1).contiguous()
    l32 = lsh.to(torch.int32).contiguous()
    is_cross = self_idx is None
    s32 = None
    if not is_cross:
        s32 = self_idx.to(torch.int32).expand(B, H, N).contiguous()
    # true_max_idx: one maximum over the whole combined tensor (:1031), kept
    # on the device (no host sync).
    parts = [l32.max()]
    if Kw:
        parts.append(win32.max())
    if g.numel():
        parts.append(g.max())
    true_max = torch.stack(parts).max().reshape(1).contiguous()
    p = GraphParams()
    p.B, p.H, p.N, p.A, p.K, p.G = B, H, N, A, total_k, g.numel()
    p.causal, p.is_cross = 0, int(is_cross)
    kall = Kw + g.numel() + A
    W = min(total_k, kall) if is_cross else min(total_k - 1, kall) + 1
    dev = lsh.device
    nb = torch.empty((B, H, N, W), dtype=torch.int32, device=dev)
    valid = torch.empty((B, H, N, W), dtype=torch.uint8, device=dev)
    check(_lib.load().ssa_merge(ctypes.byref(p), _ptr(l32), _ptr(g), _ptr(win32) if Kw else None,
                                Kw, _ptr(s32), _ptr(true_max), _ptr(nb), _ptr(valid), _stream(dev)),
          "ssa_merge")
    return nb, valid


def hash_ids(x: torch.Tensor, rand_proj: torch.Tensor, R: int, max_p: int, p_eff: int):
    """Per-round bucket ids of x (B, heads, rows, d): (B*heads, R, rows) int32."""
    _require_cuda(x, rand_proj)
    x, sb, sh, sn = _rows(x)
    B, Hh, Nr, d = x.shape
    rp = rand_proj.detach().to(torch.float32).contiguous()
    out = torch.empty((B * Hh, R, Nr), dtype=torch.int32, device=x.device)
    check(_lib.load().ssa_hash_ids(_ptr(x), _dtype_code(x), B, Hh, Nr, d, sb, sh, sn, _ptr(rp), R,
                                   max_p, p_eff, _ptr(out), _stream(x.device)), "ssa_hash_ids")
    return out


def _attn_params(q, k, v, nb, scale, fp32w, o_strides):
    B, H, N, d = q.shape
    _, n_kv, M, _ = k.shape
    if v.shape != k.shape:
        raise ValueError(f"k {tuple(k.shape)} and v {tuple(v.shape)} differ")
    if nb.shape[:3] != (B, H, N):
        raise ValueError(f"neighbors {tuple(nb.shape)} do not match q {tuple(q.shape)}")
    p = AttnParams()
    p.B, p.H, p.n_kv, p.N, p.M, p.d, p.Kn = B, H, n_kv, N, M, d, nb.shape[3]
    p.dtype = _dtype_code(q)
    p.nb_i64 = int(nb.dtype == torch.int64)
    p.fp32_weights = int(bool(fp32w))
    p.scale = float(scale)
    p.o_sb, p.o_sh, p.o_sn = o_strides
    return p


def _index_inputs(nb, valid):
    if nb.dtype not in (torch.int32, torch.int64):
        nb = nb.to(torch.int32)
    nb = nb.contiguous()
    if valid.dtype == torch.bool:
        valid = valid.contiguous().view(torch.uint8)
    else:
        valid = valid.to(torch.uint8).contiguous()
    return nb, valid


def _set_dropout(p, dropout):
    """dropout: None, or (p, seed, offset) -- the Philox key and counter offset
    of the keep decisions (the same triple must reach the backward)."""
    if dropout is not None and dropout[0] > 0.0:
        p.dropout_p = float(dropout[0])
        p.dropout_seed = int(dropout[1]) & 0xFFFFFFFFFFFFFFFF
        p.dropout_offset = int(dropout[2]) & 0xFFFFFFFFFFFFFFFF


def new_dropout_key(p: float):
    """(p, seed, offset) for one dropout application: a 62-bit seed drawn from
    torch's default generator, so torch.manual_seed makes it reproducible and
    every call draws a fresh mask."""
    return (float(p), int(torch.randint(0, 2 ** 62, (1,)).item()), 0)


def attn_fwd(q, k, v, nb, valid, scale: float, fp32w: bool, out: Optional[torch.Tensor] = None,
             want_lse: bool = True, dropout=None):
    """Gather attention forward. `out` (B,H,N,d) may be a strided view (for
    example of a (B,N,H,d) buffer); returns (out, lse). dropout: None or
    (p, seed, offset) -- attention-weight dropout."""
    _require_cuda(q, k, v, nb, valid)
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k, v must share one dtype")
    q, *qs = _rows(q)
    k, *ks = _rows(k)
    v, *vs = _rows(v)
    nb, valid = _index_inputs(nb, valid)
    B, H, N, d = q.shape
    if out is None:
        out = torch.empty((B, N, H, d), dtype=q.dtype, device=q.device).permute(0, 2, 1, 3)
    o = out.stride()
    p = _attn_params(q, k, v, nb, scale, fp32w, (o[0], o[1], o[2]))
    _set_dropout(p, dropout)
    p.q_sb, p.q_sh, p.q_sn = qs
    p.k_sb, p.k_sh, p.k_sm = ks
    p.v_sb, p.v_sh, p.v_sm = vs
    lse = torch.empty((B, H, N), dtype=torch.float32, device=q.device) if want_lse else None
    check(_lib.load().ssa_attn_fwd(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(nb), _ptr(valid),
                                   _ptr(out), _ptr(lse), _stream(q.device)), "ssa_attn_fwd")
    return out, lse


class GraphCSR:
    """Holder of one graph's inverted neighbor index (ssa_attn_build_csr): the
    first backward that gets it builds the index, every later backward on
    the same (neighbors, valid) reuses it -- the layers of a
    CachedGraphSparseTransformer group share one."""

    def __init__(self):
        self.buf = None
        self.key = None


def attn_bwd(q, k, v, nb, valid, dO, lse, scale: float, fp32w: bool, dropout=None,
             csr: Optional[GraphCSR] = None):
    """Gradients of sum(out * dO): dq (B,H,N,d), dk/dv (B,n_kv,M,d).
    dropout: the (p, seed, offset) the forward used, or None. csr: a
    GraphCSR shared by the backward passes over one graph, or None (the
    index is then built inside this call)."""
    _require_cuda(q, k, v, nb, valid, dO, lse)
    q, *qs = _rows(q)
    k, *ks = _rows(k)
    v, *vs = _rows(v)
    dO = dO.to(q.dtype)
    dO, *os_ = _rows(dO)
    nb, valid = _index_inputs(nb, valid)
    dq = torch.empty_strided(dO.shape, dO.stride(), dtype=q.dtype, device=q.device)
    dk = torch.empty(k.shape, dtype=q.dtype, device=q.device)
    dv = torch.empty(v.shape, dtype=q.dtype, device=q.device)
    p = _attn_params(q, k, v, nb, scale, fp32w, tuple(os_))
    _set_dropout(p, dropout)
    p.q_sb, p.q_sh, p.q_sn = qs
    p.k_sb, p.k_sh, p.k_sm = ks
    p.v_sb, p.v_sh, p.v_sm = vs
    L = _lib.load()
    ws_bytes = L.ssa_attn_bwd_workspace_size(ctypes.byref(p))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    st = _stream(q.device)
    if csr is None:
        check(L.ssa_attn_bwd(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(nb), _ptr(valid), _ptr(dO),
                             _ptr(lse.contiguous()), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(ws), ws_bytes, st),
              "ssa_attn_bwd")
        return dq, dk, dv
    key = (tuple(nb.shape), nb.dtype, nb.data_ptr(), valid.data_ptr(), k.shape[1], k.shape[2])
    if csr.buf is None or csr.key != key:
        nbytes = L.ssa_attn_csr_size(ctypes.byref(p))
        csr.buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
        check(L.ssa_attn_build_csr(ctypes.byref(p), _ptr(nb), _ptr(valid), _ptr(csr.buf), nbytes, _ptr(ws),
                                   ws_bytes, st), "ssa_attn_build_csr")
        csr.key = key
    check(L.ssa_attn_bwd_csr(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(nb), _ptr(valid), _ptr(dO),
                             _ptr(lse.contiguous()), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(csr.buf),
                             csr.buf.numel(), _ptr(ws), ws_bytes, st), "ssa_attn_bwd_csr")
    return dq, dk, dv


class GatherAttention(torch.autograd.Function):
    """Autograd wrapper: the graph (nb, valid) is non-differentiable, as in
    the reference (routing decisions are sign tests and top-k)."""

    @staticmethod
    def forward(ctx, q, k, v, nb, valid, scale, fp32w, dropout=None, csr=None):
        out, lse = attn_fwd(q, k, v, nb, valid, scale, fp32w, dropout=dropout)
        ctx.save_for_backward(q, k, v, nb, valid, lse)
        ctx.scale, ctx.fp32w, ctx.dropout, ctx.csr = scale, fp32w, dropout, csr
        ctx.mark_non_differentiable()
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, nb, valid, lse = ctx.saved_tensors
        dq, dk, dv = attn_bwd(q, k, v, nb, valid, dout, lse, ctx.scale, ctx.fp32w, dropout=ctx.dropout,
                              csr=ctx.csr)
        return dq, dk, dv, None, None, None, None, None, None


def gather_attention(q, k, v, nb, valid, scale: float, fp32w: bool = False, dropout=None,
                     csr: Optional[GraphCSR] = None):
    """dropout: None or (p, seed, offset); see new_dropout_key. csr: a
    GraphCSR that the backward passes over this graph share."""
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return GatherAttention.apply(q, k, v, nb, valid, scale, fp32w, dropout, csr)
    return attn_fwd(q, k, v, nb, valid, scale, fp32w, want_lse=False, dropout=dropout)[0]


def neighbor_overlap(nb_a: torch.Tensor, nb_b: torch.Tensor, valid_a: torch.Tensor,
                     valid_b: torch.Tensor) -> torch.Tensor:
    """Per-row Jaccard similarity of two (..., K) neighbor-set tensors on the
    GPU; returns fp32 of shape nb_a.shape[:-1]."""
    _require_cuda(nb_a, nb_b, valid_a, valid_b)
    if nb_a.shape != nb_b.shape or valid_a.shape != nb_a.shape or valid_b.shape != nb_a.shape:
        raise ValueError("neighbor_overlap: all four tensors must have one shape")
    K = nb_a.shape[-1]
    rows = nb_a.numel() // K
    i64 = nb_a.dtype == torch.int64 or nb_b.dtype == torch.int64
    dt = torch.int64 if i64 else torch.int32
    a = nb_a.to(dt).contiguous()
    b = nb_b.to(dt).contiguous()
    va = valid_a.to(torch.uint8).contiguous()
    vb = valid_b.to(torch.uint8).contiguous()
    out = torch.empty(nb_a.shape[:-1], dtype=torch.float32, device=nb_a.device)
    check(_lib.load().ssa_neighbor_overlap(_ptr(a), _ptr(va), _ptr(b), _ptr(vb), rows, K, int(i64),
                                           _ptr(out), _stream(nb_a.device)), "ssa_neighbor_overlap")
    return out


class graph_profile:
    """Context manager: graph builds inside it record per-stage CUDA events
    (ssa_graph_profile); `times()` returns {stage: ms} of the most recent
    build, waiting for it to finish."""

    def __enter__(self):
        check(_lib.load().ssa_graph_profile(1), "ssa_graph_profile")
        return self

    def times(self):
        buf = (ctypes.c_float * len(_lib.GRAPH_STAGES))()
        check(_lib.load().ssa_graph_stage_times(buf), "ssa_graph_stage_times")
        return dict(zip(_lib.GRAPH_STAGES, [float(x) for x in buf]))

    def __exit__(self, *exc):
        _lib.load().ssa_graph_profile(0)
        return False
