"""The reference's Python API over the sm_100a kernels.

Same class and function names, constructor arguments, parameter/buffer
names, RNG consumption order and return contracts as daedalus/SSA's
`sparse_attention.py`, so models, checkpoints (`state_dict`) and callers move
over unchanged. The hot path -- `build_graph` and `apply_graph` (and
`forward`, which calls them) -- runs only on CUDA tensors, through
libssa_b200.so; calling it with CPU tensors raises.

Internally `forward` hands the kernels the (B, N, H*d) projection outputs as
strided (B, H, N, d) views, keeps K/V unexpanded (B, n_kv, M, d) for GQA/MQA,
and writes attention output directly in the (B, N, H, d) layout that the
output projection reads, so no transpose, `repeat_interleave` or int64
neighbor tensor is materialised. The public `build_graph` / `_split_kv`
keep the reference's int64/bool and expanded-head contracts.
"""
from __future__ import annotations

import math
import warnings
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops


# ---------------------------------------------------------------------------
# Config (sparse_attention.py:188-285)
# ---------------------------------------------------------------------------
@dataclass
class SSAConfig:
    d_model: int = 512
    num_heads: int = 8
    num_kv_heads: Optional[int] = None
    num_neighbors: int = 128
    max_num_hashes: int = 12
    num_hash_rounds: int = 8
    lsh_num_probes: int = 0
    window_size: int = 8
    num_global_tokens: int = 2
    global_token_indices: Optional[list] = None
    dropout: float = 0.0
    causal: bool = False
    fp32_attn_weights: bool = False


# ---------------------------------------------------------------------------
# Regime tracker (sparse_attention.py:292-350): opt-in bookkeeping.
# ---------------------------------------------------------------------------
class SubquadraticRegimeTracker:
    """Records (N, K, R, C) per call; `check` reports whether K, R and C
    stayed constant across calls (the regime in which the build is
    sub-quadratic in N) and warns otherwise."""

    def __init__(self):
        self.history: list = []

    def record(self, N: int, K: int, R: int, C: int) -> None:
        self.history.append((N, K, R, C))

    def check(self, warn: bool = True) -> bool:
        if len(self.history) < 2:
            return True
        Ks = {h[1] for h in self.history}
        Rs = {h[2] for h in self.history}
        Cs = {h[3] for h in self.history}
        ok = len(Ks) == 1 and len(Rs) == 1 and len(Cs) == 1
        if not ok and warn:
            ns = [h[0] for h in self.history]
            warnings.warn(
                f"SubquadraticRegimeTracker: K/R/C varied across {len(self.history)} calls "
                f"(N ranged {min(ns)}-{max(ns)}, K values seen: {sorted(Ks)}, R values: "
                f"{sorted(Rs)}, C values: {sorted(Cs)}). Sub-quadratic cost only holds when "
                f"K, R and C do not grow with N.", stacklevel=2)
        return ok


# ---------------------------------------------------------------------------
# Window / global index builders (sparse_attention.py:357-415)
# ---------------------------------------------------------------------------
class WindowGraphBuilder(nn.Module):
    """Query i attends keys i-w..i+w clamped to [0, M-1]; causal maps the
    future offsets to i. Returns (N, 2w+1) int64. Inside `build_graph` the
    window is generated in-kernel; this module serves callers that compose
    the builders themselves."""

    def __init__(self, window_size: int, causal: bool = False):
        super().__init__()
        self.w = window_size
        self.causal = causal

    def forward(self, N: int, M: int, device) -> torch.Tensor:
        pos = torch.arange(N, device=device)
        off = torch.arange(-self.w, self.w + 1, device=device)
        idx = pos.unsqueeze(1) + off.unsqueeze(0)
        if self.causal:
            idx = torch.where((off > 0).unsqueeze(0), pos.unsqueeze(1), idx)
        return idx.clamp(0, M - 1)


class GlobalGraphBuilder(nn.Module):
    """Keys seen by every query: arange(min(G, M)) or explicit indices
    clamped to [0, M-1] (order and duplicates kept)."""

    def __init__(self, num_global: int, indices: Optional[list] = None):
        super().__init__()
        if indices is not None:
            self.register_buffer("_fixed_idx", torch.tensor(indices, dtype=torch.long),
                                 persistent=False)
            self.G = len(indices)
            self._use_fixed = True
        else:
            self.G = num_global
            self._use_fixed = False

    def forward(self, M: int, device) -> torch.Tensor:
        if self._use_fixed:
            return self._fixed_idx.to(device).clamp(0, M - 1)
        return torch.arange(min(self.G, M), device=device)


# ---------------------------------------------------------------------------
# LSH builder (sparse_attention.py:422-959)
# ---------------------------------------------------------------------------
class LSHGraphBuilder(nn.Module):
    """Multi-round random-hyperplane LSH candidate selection.

    `rand_proj` (R, max_num_hashes, d) is a persistent fp32 buffer and stays
    fp32 when the module is cast (`.to(torch.bfloat16)`), so hashing is
    always an fp32 sign test. `forward` runs the whole selection on the GPU
    (hash, bucket, multi-probe, rescore, top-k, fallbacks)."""

    def __init__(self, d_head: int, lsh_candidates: int, num_rounds: int = 1,
                 max_num_hashes: int = 12, num_probes: int = 0):
        super().__init__()
        assert max_num_hashes <= 12, (
            f"max_num_hashes={max_num_hashes}: bucket tables grow as 2**P per round; "
            f"use more num_hash_rounds instead of more planes")
        self.max_P = max_num_hashes
        self.C = lsh_candidates
        self.R = num_rounds
        assert num_probes >= 0, f"num_probes must be >= 0, got {num_probes}"
        self.T = num_probes
        projs = []
        for _ in range(num_rounds):  # same RNG consumption as the reference (:511-519)
            p = torch.randn(max_num_hashes, d_head)
            p = p / p.norm(dim=-1, keepdim=True).clamp_min(1e-12)
            projs.append(p)
        self.register_buffer("rand_proj", torch.stack(projs))

    def _apply(self, fn, recurse=True):
        keep = self.rand_proj
        super()._apply(fn, recurse)
        if self.rand_proj.dtype != torch.float32:
            self.rand_proj = keep.to(device=self.rand_proj.device, dtype=torch.float32)
        return self

    @staticmethod
    def compute_effective_p(M: int, C: int, max_p: int, min_p: int = 1) -> int:
        """round(log2(M / C)) clamped to [min_p, max_p] (Python round)."""
        if M <= 1 or C <= 0:
            return min_p
        return max(min_p, min(max_p, round(math.log2(max(M, 1) / max(C, 1)))))

    def _hash(self, x: torch.Tensor, round_idx: int, p_eff: int) -> torch.Tensor:
        """Bucket ids (...,) of x (..., d) in round `round_idx` (GPU kernel)."""
        lead = x.shape[:-1]
        x4 = x.reshape(1, 1, -1, x.shape[-1])
        rp = self.rand_proj[round_idx:round_idx + 1]
        ids = ops.hash_ids(x4, rp, 1, self.max_P, p_eff)
        return ids.reshape(lead).long()

    def _hash_proj(self, x: torch.Tensor, round_idx: int, p_eff: int) -> torch.Tensor:
        """Hyperplane projections (..., p_eff) in fp32 (diagnostic helper)."""
        return x.float() @ self.rand_proj[round_idx, :p_eff].T

    def _probe_ids(self, proj: torch.Tensor, p_eff: int, num_probes: int) -> list:
        """Multi-probe bucket ids: probe t flips the bit with the t-th smallest
        |proj| of the original id (diagnostic helper; the kernels compute
        the same ids in registers)."""
        num_probes = min(num_probes, p_eff)
        if num_probes <= 0:
            return []
        bits = (proj > 0).long()
        powers = 2 ** torch.arange(p_eff, device=proj.device)
        base = (bits * powers).sum(-1)
        order = proj.abs().argsort(dim=-1, stable=True)
        return [base ^ powers[order[..., t]] for t in range(num_probes)]

    def output_width(self, M: int, top_k: int) -> int:
        p_eff = self.compute_effective_p(M, self.C, self.max_P)
        return min(top_k, self.R * self.C * (1 + min(self.T, p_eff)))

    def forward(self, q: torch.Tensor, k: torch.Tensor, top_k: int, causal: bool = False,
                glob_fallback: Optional[torch.Tensor] = None) -> torch.Tensor:
        """(B, H, N, A) int64: per query the top-A candidate keys by q.k over
        the union of the R rounds' buckets, in descending score order, with
        the reference's fallback slots last. k may be (B, H, M, d) or the
        unexpanded (B, n_kv, M, d)."""
        M = k.shape[2]
        p_eff = self.compute_effective_p(M, self.C, self.max_P)
        A = self.output_width(M, top_k)
        if glob_fallback is None:
            glob_fallback = torch.zeros(1, dtype=torch.long, device=q.device)
        out = ops.lsh_select(q, k, self.rand_proj, glob_fallback, R=self.R, max_p=self.max_P,
                             p_eff=p_eff, C=self.C, T=self.T, A=A, causal=bool(causal))
        return out.long()


# ---------------------------------------------------------------------------
# merge_neighbors (sparse_attention.py:966-1089)
# ---------------------------------------------------------------------------
def merge_neighbors(win_idx: torch.Tensor, glob_idx: torch.Tensor, lsh_idx: torch.Tensor,
                    self_idx: Optional[torch.Tensor], total_k: int, N: int, B: int, H: int,
                    device) -> Tuple[torch.Tensor, torch.Tensor]:
    """Union of window, global and LSH indices per (b, h, query): self (if
    given) in slot 0, then the ascending unique remaining indices, then
    padding (index 0, valid False). Returns int64 neighbors and bool valid."""
    nb, valid = ops.merge(win_idx.to(lsh_idx.device), glob_idx.to(lsh_idx.device), lsh_idx,
                          self_idx, total_k)
    return nb.long(), valid.view(torch.bool)  # 0 / 1 bytes: a view, no copy


# ---------------------------------------------------------------------------
# sparse_gather_attention (sparse_attention.py:1096-1199)
# ---------------------------------------------------------------------------
def sparse_gather_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            neighbors: torch.Tensor, scale: float,
                            valid: Optional[torch.Tensor] = None, dropout: float = 0.0,
                            training: bool = False, fp32_attn_weights: bool = False) -> torch.Tensor:
    """(B, H, N, d): softmax over the neighbor slots of fp32 q.k * scale
    (invalid slots masked), weights cast to the value dtype unless
    fp32_attn_weights, weighted sum of the neighbor value rows. k, v may be
    (B, H, M, d) or unexpanded (B, n_kv, M, d)."""
    if valid is None:
        valid = torch.ones(neighbors.shape, dtype=torch.bool, device=neighbors.device)
    # F.dropout on the attention weights after their cast (:1193-1194): the
    # keep mask comes from an in-kernel counter-based generator keyed by a
    # seed drawn here, and the backward recomputes the same mask.
    drop = ops.new_dropout_key(dropout) if (dropout > 0.0 and training) else None
    return ops.gather_attention(q, k, v, neighbors, valid, scale, fp32_attn_weights, dropout=drop)


# ---------------------------------------------------------------------------
# SparseAttention (sparse_attention.py:1206-1510)
# ---------------------------------------------------------------------------
class _FusedQKVHash(torch.autograd.Function):
    """x -> qkv = x [Wq; Wk; Wv]^T (B, N, (H + 2 n_kv) d) through the fused
    projection + hash kernel; its graph state goes to state[0] (None, and a
    plain matmul, when the kernel does not serve the shapes). Backward: the
    projection's gradients (dx = dqkv W, dW = dqkv^T x)."""

    @staticmethod
    def forward(ctx, x, wq, wk, wv, attn, causal, state):
        w = torch.cat([wq, wk, wv], dim=0)
        lsh = attn.lsh_builder
        N = x.shape[1]
        res = ops.qkv_project_hash(x, w, lsh.rand_proj, attn._glob(N, x.device), H=attn.H, n_kv=attn.n_kv,
                                   R=lsh.R, max_p=lsh.max_P, p_eff=lsh.compute_effective_p(N, lsh.C, lsh.max_P),
                                   C=lsh.C, T=lsh.T, A=lsh.output_width(N, attn.lsh_k), causal=causal,
                                   K=attn.K, window=attn.config.window_size)
        if res is None:
            qkv = torch.nn.functional.linear(x, w)
            state.append(None)
        else:
            qkv = res[0]
            state.append(res[1])
        ctx.save_for_backward(x, w)
        ctx.splits = (wq.shape[0], wk.shape[0], wv.shape[0])
        return qkv

    @staticmethod
    def backward(ctx, gq):
        x, w = ctx.saved_tensors
        dx = gq @ w
        dw = gq.reshape(-1, gq.shape[-1]).t() @ x.reshape(-1, x.shape[-1])
        dwq, dwk, dwv = torch.split(dw, ctx.splits, dim=0)
        return dx, dwq, dwk, dwv, None, None, None


class SparseAttention(nn.Module):
    """Sparse multi-head attention over a window + global + LSH neighbor
    graph. Self-attention (key_value None) or cross-attention (no window,
    no self slot, never causal)."""

    def __init__(self, config: SSAConfig):
        super().__init__()
        assert config.d_model % config.num_heads == 0, \
            f"d_model ({config.d_model}) must be divisible by num_heads ({config.num_heads})"
        n_kv = config.num_kv_heads if config.num_kv_heads is not None else config.num_heads
        assert config.num_heads % n_kv == 0, \
            f"num_heads ({config.num_heads}) must be divisible by num_kv_heads ({n_kv})"
        self.config = config
        self.H = config.num_heads
        self.n_kv = n_kv
        self.kv_rep = config.num_heads // n_kv
        self.d_head = config.d_model // config.num_heads
        self.K = config.num_neighbors
        self.scale = self.d_head ** -0.5
        # Same construction order as the reference, so one seed gives the same weights.
        self.Wq = nn.Linear(config.d_model, config.num_heads * self.d_head, bias=False)
        self.Wk = nn.Linear(config.d_model, n_kv * self.d_head, bias=False)
        self.Wv = nn.Linear(config.d_model, n_kv * self.d_head, bias=False)
        self.Wo = nn.Linear(config.num_heads * self.d_head, config.d_model, bias=False)
        self.win_builder = WindowGraphBuilder(config.window_size, config.causal)
        self.glob_builder = GlobalGraphBuilder(num_global=config.num_global_tokens,
                                               indices=config.global_token_indices)
        n_glob = (len(config.global_token_indices) if config.global_token_indices is not None
                  else config.num_global_tokens)
        guaranteed = 2 * config.window_size + 1 + n_glob + 1
        self.lsh_k = max(self.K - guaranteed, 8)
        if guaranteed > self.K:
            warnings.warn(
                f"SSAConfig: window+global+self budget ({guaranteed}) exceeds num_neighbors "
                f"({self.K}). lsh_k is floored at 8 and a large fraction of computed candidates "
                f"will be discarded as padding.", stacklevel=2)
        self.lsh_builder = LSHGraphBuilder(d_head=self.d_head, max_num_hashes=config.max_num_hashes,
                                           lsh_candidates=self.lsh_k * 4,
                                           num_rounds=config.num_hash_rounds,
                                           num_probes=config.lsh_num_probes)
        self.dp = config.dropout
        self._glob_cache = {}
        # bf16 self-attention: True routes Wq / Wk / Wv through the fused QKV
        # projection + hash kernel (ssa_qkv_proj_hash) where it serves the
        # shapes. Off by default: cuBLAS's GEMM plus the tensor-core hash is
        # faster today.
        self.fuse_qkv = False

    # -- layout helpers (sparse_attention.py:1300-1323) ----------------------
    def _split_q(self, x):
        B, N, _ = x.shape
        return x.view(B, N, self.H, self.d_head).transpose(1, 2)

    def _split_kv(self, x):
        B, M, _ = x.shape
        kv = x.view(B, M, self.n_kv, self.d_head).transpose(1, 2)
        if self.kv_rep > 1:
            kv = kv.repeat_interleave(self.kv_rep, dim=1)
        return kv

    def _split(self, x):
        return self._split_q(x)

    def _merge(self, x):
        B, H, N, _ = x.shape
        return x.transpose(1, 2).contiguous().view(B, N, self.config.d_model)

    def _split_kv_grouped(self, x):
        """(B, M, n_kv*d) -> (B, n_kv, M, d) view: the kernels map head h to
        kv head h // kv_rep themselves."""
        B, M, _ = x.shape
        return x.view(B, M, self.n_kv, self.d_head).transpose(1, 2)

    def _glob(self, M: int, device) -> torch.Tensor:
        key = (M, str(device))
        g = self._glob_cache.get(key)
        if g is None:
            g = self.glob_builder(M, device).to(torch.int32)
            self._glob_cache[key] = g
        return g

    def _graph(self, q, k, M: int, causal: bool, is_cross: bool, q_row0: int = 0):
        """Neighbor graph as int32 neighbors + uint8 valid (internal form).
        q_row0: sequence position of q's first row (query-row sharding)."""
        lsh = self.lsh_builder
        p_eff = lsh.compute_effective_p(M, lsh.C, lsh.max_P)
        A = lsh.output_width(M, self.lsh_k)
        return ops.build_graph(q, k, lsh.rand_proj, self._glob(M, q.device), R=lsh.R,
                               max_p=lsh.max_P, p_eff=p_eff, C=lsh.C, T=lsh.T, A=A,
                               causal=causal, is_cross=is_cross, K=self.K,
                               window=self.config.window_size, q_row0=q_row0)

    def build_graph(self, q: torch.Tensor, k: torch.Tensor, N: int, M: int, B: int, device,
                    causal: bool, is_cross: bool) -> Tuple[torch.Tensor, torch.Tensor]:
        """(neighbors int64, valid bool), both (B, H, N, K): window + global +
        LSH + self, merged and deduplicated."""
        nb, valid = self._graph(q, k, M, bool(causal) and not is_cross, is_cross)
        return nb.long(), valid.view(torch.bool)  # 0 / 1 bytes: a view, no copy

    def apply_graph(self, q, k, v, neighbors, valid) -> torch.Tensor:
        return sparse_gather_attention(q, k, v, neighbors, scale=self.scale, valid=valid,
                                       dropout=self.dp, training=self.training,
                                       fp32_attn_weights=self.config.fp32_attn_weights)

    def forward(self, x: torch.Tensor, key_value: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None,
                return_stats: bool = False) -> Tuple[torch.Tensor, dict]:
        if attention_mask is not None:
            raise ValueError(
                "SparseAttention does not accept an external attention_mask. Use "
                "config.causal=True for autoregressive masking (handled by the graph "
                "builders). For padding, zero out padding positions in x before calling "
                "forward(), or set num_global_tokens to 0 so padding tokens are not forced "
                "into every query's neighbor set.")
        B, N, _ = x.shape
        is_cross = key_value is not None
        src = key_value if is_cross else x
        M = src.shape[1]
        causal = self.config.causal and not is_cross
        fused = None
        if not is_cross and x.dtype == torch.bfloat16 and self.fuse_qkv:
            # One tcgen05 GEMM for Wq / Wk / Wv whose epilogue also hashes q
            # and k for the graph (None when the shapes are not served).
            state = []
            qkv = _FusedQKVHash.apply(x, self.Wq.weight, self.Wk.weight, self.Wv.weight, self, causal, state)
            if state[0] is not None:
                q, k, v = ops.split_qkv(qkv, self.H, self.n_kv)
                nb, valid = ops.build_graph_prehashed(q, k, state[0])
                fused = True
        if fused is None:
            q = self._split_q(self.Wq(x))
            k = self._split_kv_grouped(self.Wk(src))
            v = self._split_kv_grouped(self.Wv(src))
            nb, valid = self._graph(q, k, M, causal, is_cross)
        drop = ops.new_dropout_key(self.dp) if (self.dp > 0.0 and self.training) else None
        out = ops.gather_attention(q, k, v, nb, valid, self.scale, self.config.fp32_attn_weights,
                                   dropout=drop)
        out_proj = self.Wo(out.transpose(1, 2).reshape(B, N, self.H * self.d_head))
        if not return_stats:
            return out_proj, {}
        peak_sparse = B * self.H * N * self.K * self.d_head
        peak_full = B * self.H * N * M * self.d_head
        stats = {
            "neighbors_shape": tuple(nb.shape),
            "peak_sparse_elems": peak_sparse,
            "peak_full_elems": peak_full,
            "compression": peak_full / peak_sparse,
            "padding_fraction": (valid == 0).float().mean().item(),
        }
        return out_proj, stats


# ---------------------------------------------------------------------------
# Transformer stacks (sparse_attention.py:1517-1550, :1688-1792)
# ---------------------------------------------------------------------------
class SparseTransformerLayer(nn.Module):
    """Pre-LN residual block: x + attn(LN1 x) + FF(LN2(x + attn))."""

    def __init__(self, config: SSAConfig, ffn_mult: int = 4):
        super().__init__()
        d = config.d_model
        self.attn = SparseAttention(config)
        self.ff = nn.Sequential(nn.Linear(d, d * ffn_mult), nn.GELU(), nn.Dropout(config.dropout),
                                nn.Linear(d * ffn_mult, d), nn.Dropout(config.dropout))
        self.norm1 = nn.LayerNorm(d)
        self.norm2 = nn.LayerNorm(d)

    def forward(self, x, return_stats: bool = False):
        a, stats = self.attn(self.norm1(x), return_stats=return_stats)
        return x + a + self.ff(self.norm2(x + a)), stats


class SparseTransformer(nn.Module):
    def __init__(self, config: SSAConfig, num_layers: int = 6, vocab_size: int = 0):
        super().__init__()
        self.embed = nn.Embedding(vocab_size, config.d_model) if vocab_size else None
        self.layers = nn.ModuleList([SparseTransformerLayer(config) for _ in range(num_layers)])
        self.norm = nn.LayerNorm(config.d_model)

    def forward(self, x, return_stats: bool = False):
        if self.embed is not None:
            x = self.embed(x)
        stats_list = []
        for layer in self.layers:
            x, stats = layer(x, return_stats=return_stats)
            stats_list.append(stats)
        return self.norm(x), stats_list


def neighbor_overlap(neighbors_a: torch.Tensor, neighbors_b: torch.Tensor,
                     valid_a: torch.Tensor, valid_b: torch.Tensor) -> torch.Tensor:
    """Per-(b, h, query) Jaccard similarity of two neighbor sets, padding
    ignored (diagnostic, sparse_attention.py:1583-1615), as one CUDA kernel:
    no (B, H, N, K, K) match tensor."""
    return ops.neighbor_overlap(neighbors_a, neighbors_b, valid_a, valid_b)


def measure_cross_layer_overlap(model: "SparseTransformer", x: torch.Tensor) -> dict:
    """Adjacent-layer neighbor-graph overlap of a SparseTransformer
    (diagnostic, sparse_attention.py:1618-1685)."""
    h = model.embed(x) if model.embed is not None else x
    graphs = []
    for layer in model.layers:
        normed = layer.norm1(h)
        attn = layer.attn
        B, N, _ = normed.shape
        q = attn._split_q(attn.Wq(normed))
        k = attn._split_kv_grouped(attn.Wk(normed))
        v = attn._split_kv_grouped(attn.Wv(normed))
        nb, valid = attn._graph(q, k, N, attn.config.causal, False)
        graphs.append((nb.long(), valid.view(torch.bool)))
        out = ops.gather_attention(q, k, v, nb, valid, attn.scale, attn.config.fp32_attn_weights)
        a = attn.Wo(out.transpose(1, 2).reshape(B, N, attn.H * attn.d_head))
        h = h + a + layer.ff(layer.norm2(h + a))
    overlaps = [neighbor_overlap(graphs[i][0], graphs[i + 1][0], graphs[i][1], graphs[i + 1][1])
                for i in range(len(graphs) - 1)]
    return {"per_pair_overlap": overlaps,
            "mean_overlap_per_adjacent_pair": [ov.mean().item() for ov in overlaps],
            "num_layers": len(model.layers)}


class CachedGraphSparseTransformer(nn.Module):
    """Builds the neighbor graph once per group of `reuse_every` layers (with
    that group's shared builder) and reuses it for the group's other layers,
    each applying it to its own q/k/v."""

    def __init__(self, config: SSAConfig, num_layers: int, reuse_every: int = 4,
                 ffn_mult: int = 4):
        super().__init__()
        assert reuse_every >= 1
        self.reuse_every = reuse_every
        self.config = config
        num_groups = math.ceil(num_layers / reuse_every)
        self.shared_attn_per_group = nn.ModuleList([SparseAttention(config) for _ in range(num_groups)])
        self.group_of = [i // reuse_every for i in range(num_layers)]
        self.layers = nn.ModuleList([SparseTransformerLayer(config, ffn_mult) for _ in range(num_layers)])
        self.norm = nn.LayerNorm(config.d_model)

    def forward(self, x, return_stats: bool = False):
        h = x
        stats_list = []
        cached, cached_group, csr = None, None, None
        for i, layer in enumerate(self.layers):
            group = self.group_of[i]
            recompute = group != cached_group
            normed = layer.norm1(h)
            attn = layer.attn
            B, N, _ = normed.shape
            q = attn._split_q(attn.Wq(normed))
            k = attn._split_kv_grouped(attn.Wk(normed))
            v = attn._split_kv_grouped(attn.Wv(normed))
            if recompute:
                cached = self.shared_attn_per_group[group]._graph(q, k, N, attn.config.causal, False)
                cached_group = group
                csr = ops.GraphCSR()  # the group's backward passes build its inverted index once
            nb, valid = cached
            drop = ops.new_dropout_key(attn.dp) if (attn.dp > 0.0 and attn.training) else None
            out = ops.gather_attention(q, k, v, nb, valid, attn.scale, attn.config.fp32_attn_weights,
                                       dropout=drop, csr=csr)
            a = attn.Wo(out.transpose(1, 2).reshape(B, N, attn.H * attn.d_head))
            h = h + a + layer.ff(layer.norm2(h + a))
            if return_stats:
                peak_sparse = B * attn.H * N * attn.K * attn.d_head
                peak_full = B * attn.H * N * N * attn.d_head
                stats_list.append({"neighbors_shape": tuple(nb.shape),
                                   "compression": peak_full / peak_sparse,
                                   "padding_fraction": (valid == 0).float().mean().item(),
                                   "graph_recomputed": recompute})
            else:
                stats_list.append({})
        return self.norm(h), stats_list
