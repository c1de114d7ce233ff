"""Multi-GPU partitioning of the sparse-attention hot path: one process per
GPU, with torch.distributed for the plumbing.

The reference runs on one device and has no distributed code. This module
splits one job across ranks in two ways.

* **Group sharding.** Each rank owns whole (batch element, kv-head) units,
  numbered batch-major and split into contiguous ranges. A unit's graph
  build and attention read only its own q heads and its own kv head, so
  ranks exchange nothing on the hot path.
* **Query-row sharding.** This is for one long sequence. Each rank owns a
  contiguous block of query rows and projects q, k and v for those rows. It
  then receives every key and value row once, through an all-gather (NCCL
  over NVLink). Keys travel sequence-major, (rows, B, n_kv, d), so the
  gathered buffer is the whole K as a strided (B, n_kv, M, d) view, with no
  copy. The graph build sees its queries' sequence positions through
  `q_row0`, which is what makes the causal limit, the window and the self
  slot come out as in the unsharded build.

The per-slice compute (graph build and gather attention) is passed in as
functions; by default they are this package's CUDA ops.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import torch

from . import ops


def split_range(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Rank's [lo, hi) of a contiguous, near-equal split of range(total)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


@dataclass(frozen=True)
class GroupSlice:
    """kv heads [g0, g1) of batch elements [b0, b1), and the q heads that read
    them; a slice spans several batch elements only with every kv head."""
    b0: int
    b1: int
    g0: int
    g1: int


def group_slices(B: int, n_kv: int, world: int, rank: int) -> List[GroupSlice]:
    """The rank's (batch, kv-head) units as blocks: runs of consecutive kv
    heads within one batch element, and whole consecutive batch elements
    merged into one block."""
    u0, u1 = split_range(B * n_kv, world, rank)
    runs = []
    u = u0
    while u < u1:
        b, g = divmod(u, n_kv)
        g1 = min(n_kv, g + (u1 - u))
        runs.append((b, g, g1))
        u += g1 - g
    out: List[GroupSlice] = []
    for b, g0, g1 in runs:
        full = g0 == 0 and g1 == n_kv
        if full and out and out[-1].b1 == b and out[-1].g0 == 0 and out[-1].g1 == n_kv:
            out[-1] = GroupSlice(out[-1].b0, b + 1, 0, n_kv)
        else:
            out.append(GroupSlice(b, b + 1, g0, g1))
    return out


def slice_views(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, s: GroupSlice, rep: int):
    """Strided views of one slice: q (b1-b0, (g1-g0)*rep, N, d), k and v
    (b1-b0, g1-g0, M, d). q head h reads kv head h // rep."""
    return (q[s.b0:s.b1, s.g0 * rep:s.g1 * rep], k[s.b0:s.b1, s.g0:s.g1], v[s.b0:s.b1, s.g0:s.g1])


def gather_seq_major(local: torch.Tensor, group=None, async_op: bool = False):
    """All-gather of sequence-major rows: local (m, ...) from every rank,
    rank order, into one (world * m, ...) tensor. With async_op, returns
    (tensor, work); work.wait() orders later work on the current stream
    after the transfer."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    local = local.contiguous()
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    work = dist.all_gather_into_tensor(out, local, group=group, async_op=async_op)
    return (out, work) if async_op else out


def seq_major_view(x: torch.Tensor) -> torch.Tensor:
    """(M, B, n_kv, d) -> a strided (B, n_kv, M, d) view (no copy)."""
    return x.permute(1, 2, 0, 3)


GraphFn = Callable[..., Tuple[torch.Tensor, torch.Tensor]]
AttnFn = Callable[..., torch.Tensor]


def _default_graph(module):
    def graph(q, k, M, causal, is_cross, q_row0):
        return module._graph(q, k, M, causal, is_cross, q_row0=q_row0)
    return graph


def _default_attn(module):
    def attn(q, k, v, nb, valid):
        out, _ = ops.attn_fwd(q, k, v, nb, valid, module.scale, module.config.fp32_attn_weights,
                              want_lse=False)
        return out
    return attn


class GroupSharded:
    """Graph build + gather attention for a rank's share of (batch, kv-head)
    units of one job. No collective."""

    def __init__(self, module, world: int, rank: int, *, causal: bool, is_cross: bool = False,
                 graph_fn: Optional[GraphFn] = None, attn_fn: Optional[AttnFn] = None):
        self.module, self.world, self.rank = module, world, rank
        self.causal, self.is_cross = bool(causal) and not is_cross, is_cross
        self.graph_fn = graph_fn or _default_graph(module)
        self.attn_fn = attn_fn or _default_attn(module)

    def slices(self, B: int, n_kv: int) -> List[GroupSlice]:
        return group_slices(B, n_kv, self.world, self.rank)

    def step(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        """q (B,H,N,d), k/v (B,n_kv,M,d), the whole job's tensors (or views);
        returns [(slice, out (b1-b0, heads, N, d))] for this rank's slices."""
        B, H = q.shape[:2]
        n_kv, M = k.shape[1], k.shape[2]
        rep = H // n_kv
        outs = []
        for s in self.slices(B, n_kv):
            qs, ks, vs = slice_views(q, k, v, s, rep)
            nb, valid = self.graph_fn(qs, ks, M, self.causal, self.is_cross, 0)
            outs.append((s, self.attn_fn(qs, ks, vs, nb, valid)))
        return outs


class RowSharded:
    """Graph build + gather attention for a rank's block of query rows of
    one self-attention sequence, with keys and values all-gathered once."""

    def __init__(self, module, N: int, world: int, rank: int, *, causal: bool, group=None,
                 graph_fn: Optional[GraphFn] = None, attn_fn: Optional[AttnFn] = None):
        if N % world:
            raise ValueError(f"query-row sharding needs N ({N}) divisible by the world size ({world}):"
                             " every rank contributes the same number of key rows to the all-gather")
        self.module, self.N, self.world, self.rank, self.group = module, N, world, rank, group
        self.causal = bool(causal)
        self.rows = split_range(N, world, rank)
        self.graph_fn = graph_fn or _default_graph(module)
        self.attn_fn = attn_fn or _default_attn(module)

    def gather_kv(self, k_local: torch.Tensor, v_local: torch.Tensor):
        """k_local / v_local (m, B, n_kv, d) sequence-major rows of this rank
        -> full K and V as strided (B, n_kv, M, d) views."""
        return (seq_major_view(gather_seq_major(k_local, self.group)),
                seq_major_view(gather_seq_major(v_local, self.group)))

    def step(self, q_local: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor):
        """q_local (B,H,n,d) for rows [r0, r1); k_local, v_local (m,B,n_kv,d).
        Returns this rank's attention output (B,H,n,d). The values' all-gather
        runs while the graph is built; only the attention waits for it."""
        k = seq_major_view(gather_seq_major(k_local, self.group))
        v_full, v_work = gather_seq_major(v_local, self.group, async_op=True)
        nb, valid = self.graph_fn(q_local, k, self.N, self.causal, False, self.rows[0])
        v_work.wait()
        return self.attn_fn(q_local, k, seq_major_view(v_full), nb, valid)
