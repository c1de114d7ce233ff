"""Parity cases shared by the golden-fixture generator, the oracle tests and the
GPU parity tests.

Every case is a small, seeded instance of the sparse-attention hot path
(`build_graph` + `apply_graph`). Inputs are produced on the CPU with a private
`torch.Generator`, so the same case gives bit-identical q/k/v/rand_proj on any
machine running the same torch build. Cases too large to store keep only their
outputs in the fixture; the inputs are regenerated and checked by a checksum.

Shapes follow the reference hot path: q is (B, H, N, d); k and v are kept
unexpanded as (B, n_kv, M, d) and head h reads kv head h // (H // n_kv), which
is what `repeat_interleave` in `SparseAttention._split_kv` (sparse_attention.py
:1305-1315) materialises.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, asdict
from typing import List, Optional

import torch


@dataclass
class Case:
    name: str
    dtype: str                 # "fp32" or "bf16": dtype of q/k/v
    B: int
    N: int
    M: int
    H: int
    n_kv: int
    d: int
    K: int                     # num_neighbors
    w: int                     # window_size
    G: int                     # num_global_tokens (ignored when glob_idx set)
    R: int                     # num_hash_rounds
    maxP: int                  # max_num_hashes
    T: int                     # lsh_num_probes
    causal: bool
    is_cross: bool
    glob_idx: Optional[List[int]] = None
    fp32_attn_weights: bool = False
    inputs: str = "normal"     # normal | cluster | cone | zero_keys
    seed: int = 0
    store_inputs: bool = True  # False: regenerate inputs, check by checksum
    grads: bool = True

    def to_dict(self):
        return asdict(self)


# ---------------------------------------------------------------------------
# Derived quantities, restated from the reference
# ---------------------------------------------------------------------------

def derived(c: Case):
    """lsh_k, C, p_eff, T_eff, A exactly as the reference derives them.

    guaranteed / lsh_k: sparse_attention.py:1262-1266; C = 4 * lsh_k: :1294;
    p_eff: :552-557 (Python round = half to even); T_eff = min(T, p_eff):
    :629; A = min(top_k, Call): :898.
    """
    n_glob = len(c.glob_idx) if c.glob_idx is not None else c.G
    guaranteed = 2 * c.w + 1 + n_glob + 1
    lsh_k = max(c.K - guaranteed, 8)
    C = lsh_k * 4
    if c.M <= 1 or C <= 0:
        p_eff = 1
    else:
        p_eff = max(1, min(c.maxP, round(math.log2(max(c.M, 1) / max(C, 1)))))
    T_eff = min(c.T, p_eff)
    Call = c.R * C * (1 + T_eff)
    A = min(lsh_k, Call)
    return dict(lsh_k=lsh_k, C=C, p_eff=p_eff, T_eff=T_eff, Call=Call, A=A,
                n_glob=n_glob)


def glob_list(c: Case):
    """Global key indices as GlobalGraphBuilder.forward returns them
    (sparse_attention.py:411-415): explicit indices clamped to [0, M-1], or
    arange(min(G, M))."""
    if c.glob_idx is not None:
        return [min(max(g, 0), c.M - 1) for g in c.glob_idx]
    return list(range(min(c.G, c.M)))


# ---------------------------------------------------------------------------
# Deterministic inputs
# ---------------------------------------------------------------------------

def make_rand_proj(R: int, maxP: int, d: int, seed: int) -> torch.Tensor:
    """Random unit hyperplanes, (R, maxP, d) fp32, rows L2-normalised with
    clamp_min(1e-12) as in LSHGraphBuilder.__init__ (sparse_attention.py:511-520)."""
    g = torch.Generator().manual_seed(seed * 7919 + 17)
    p = torch.randn(R, maxP, d, generator=g)
    return p / p.norm(dim=-1, keepdim=True).clamp_min(1e-12)


def make_inputs(c: Case):
    """Returns q (B,H,N,d), k (B,n_kv,M,d), v (B,n_kv,M,d) in the case dtype,
    rand_proj (R,maxP,d) fp32 and dO (B,H,N,d) fp32."""
    g = torch.Generator().manual_seed(c.seed * 1000003 + 11)
    dt = torch.float32 if c.dtype == "fp32" else torch.bfloat16
    B, N, M, H, n_kv, d = c.B, c.N, c.M, c.H, c.n_kv, c.d
    if c.inputs == "normal":
        q = torch.randn(B, H, N, d, generator=g)
        k = torch.randn(B, n_kv, M, d, generator=g)
        v = torch.randn(B, n_kv, M, d, generator=g)
    elif c.inputs == "cluster":
        # 16 centres ~N(0, I), uniform assignment, +0.3 N(0, I) noise: skews
        # bucket occupancy like the long-context config's cluster mixture.
        cent = torch.randn(16, d, generator=g)
        aq = torch.randint(0, 16, (B, H, N), generator=g)
        ak = torch.randint(0, 16, (B, n_kv, M), generator=g)
        q = cent[aq] + 0.3 * torch.randn(B, H, N, d, generator=g)
        k = cent[ak] + 0.3 * torch.randn(B, n_kv, M, d, generator=g)
        v = torch.randn(B, n_kv, M, d, generator=g)
    elif c.inputs == "cone":
        # Keys in a narrow cone: most buckets stay empty, so empty-bucket
        # fallbacks, overflow pads and the invalid-first dedup rule all fire.
        axis = torch.randn(d, generator=g)
        k = axis + 0.05 * torch.randn(B, n_kv, M, d, generator=g)
        q = torch.randn(B, H, N, d, generator=g)
        v = torch.randn(B, n_kv, M, d, generator=g)
    elif c.inputs == "zero_keys":
        # All keys hash to bucket 0 (proj == 0 is not > 0); queries are ones.
        k = torch.zeros(B, n_kv, M, d)
        q = torch.ones(B, H, N, d)
        v = torch.randn(B, n_kv, M, d, generator=g)
    else:
        raise ValueError(c.inputs)
    dO = torch.randn(B, H, N, d, generator=g)
    rp = make_rand_proj(c.R, c.maxP, d, c.seed)
    return q.to(dt).contiguous(), k.to(dt).contiguous(), v.to(dt).contiguous(), rp, dO


def checksum(t: torch.Tensor) -> List[float]:
    """Cheap fingerprint used to confirm regenerated inputs are identical."""
    f = t.detach().double().reshape(-1)
    return [float(f.sum()), float((f * f).sum()), float(f[: min(64, f.numel())].abs().sum())]


# ---------------------------------------------------------------------------
# The cases
# ---------------------------------------------------------------------------

CASES: List[Case] = [
    # Scaled-down versions of the five BASELINE configs.
    Case("c1s_fp32_causal", "fp32", B=2, N=256, M=256, H=2, n_kv=2, d=64, K=64,
         w=8, G=2, R=8, maxP=12, T=0, causal=True, is_cross=False, seed=1),
    Case("c2s_bf16_gqa_causal", "bf16", B=1, N=512, M=512, H=4, n_kv=2, d=128,
         K=64, w=4, G=4, R=4, maxP=12, T=0, causal=True, is_cross=False, seed=2),
    Case("c3s_bf16_cluster_probes", "bf16", B=1, N=1024, M=1024, H=2, n_kv=2,
         d=64, K=64, w=8, G=4, R=4, maxP=12, T=2, causal=False, is_cross=False,
         inputs="cluster", seed=3),
    Case("c4s_fp32_train", "fp32", B=2, N=128, M=128, H=2, n_kv=2, d=32, K=32,
         w=3, G=2, R=4, maxP=12, T=0, causal=True, is_cross=False, seed=4),
    Case("c5s_bf16_mqa_cross", "bf16", B=2, N=128, M=512, H=4, n_kv=1, d=64,
         K=64, w=8, G=0, glob_idx=[0, 1, 300], R=4, maxP=12, T=1, causal=False,
         is_cross=True, seed=5),
    # Occupancy below C (invalid-first dedup rule) with several buckets.
    Case("occ_below_C_fp32", "fp32", B=1, N=384, M=384, H=2, n_kv=1, d=32,
         K=32, w=2, G=1, R=6, maxP=12, T=1, causal=False, is_cross=False,
         seed=6),
    # Empty buckets, pads and fallbacks.
    Case("cone_keys_causal", "fp32", B=1, N=200, M=200, H=2, n_kv=2, d=16,
         K=24, w=2, G=2, R=4, maxP=6, T=2, causal=True, is_cross=False,
         inputs="cone", seed=7),
    Case("cone_keys_cross", "bf16", B=1, N=96, M=160, H=2, n_kv=1, d=32,
         K=40, w=3, G=3, R=3, maxP=6, T=1, causal=False, is_cross=True,
         inputs="cone", seed=8),
    Case("zero_keys_fallback", "fp32", B=1, N=4, M=8, H=1, n_kv=1, d=4, K=16,
         w=1, G=2, R=1, maxP=1, T=0, causal=False, is_cross=False,
         inputs="zero_keys", seed=9, grads=False),
    # Tiny and ragged sizes (p_eff floors at 1, pool smaller than K).
    Case("tiny_n8", "fp32", B=1, N=8, M=8, H=2, n_kv=2, d=16, K=32, w=2, G=1,
         R=2, maxP=6, T=3, causal=False, is_cross=False, seed=10),
    Case("ragged_n65_causal", "fp32", B=2, N=65, M=65, H=2, n_kv=1, d=32, K=32,
         w=2, G=1, R=2, maxP=6, T=1, causal=True, is_cross=False, seed=11),
    Case("ragged_n300_bf16", "bf16", B=1, N=300, M=300, H=2, n_kv=2, d=32, K=32,
         w=2, G=1, R=2, maxP=6, T=3, causal=False, is_cross=False, seed=12),
    # Cross-attention with more queries than keys (N > M).
    Case("cross_n_gt_m", "fp32", B=1, N=10, M=3, H=1, n_kv=1, d=16, K=4, w=1,
         G=1, R=1, maxP=1, T=0, causal=False, is_cross=True, seed=13),
    # Explicit globals with duplicates and out-of-range values (clamped).
    Case("glob_dup_clamp", "fp32", B=1, N=96, M=96, H=2, n_kv=2, d=16, K=40,
         w=3, G=0, glob_idx=[5, 5, 200, 0], R=3, maxP=6, T=1, causal=True,
         is_cross=False, seed=14),
    # Window + globals exceed K: merge truncates to the smallest indices.
    Case("truncate_pool", "fp32", B=1, N=128, M=128, H=2, n_kv=2, d=32, K=16,
         w=8, G=4, R=2, maxP=6, T=0, causal=False, is_cross=False, seed=15),
    # fp32_attn_weights path in bf16.
    Case("bf16_fp32_weights", "bf16", B=1, N=256, M=256, H=4, n_kv=2, d=64,
         K=48, w=4, G=2, R=3, maxP=12, T=1, causal=True, is_cross=False,
         fp32_attn_weights=True, seed=16),
    # Full-size config 1 (fp32, MHA, causal); inputs regenerated from the seed.
    Case("c1_full", "fp32", B=2, N=1024, M=1024, H=8, n_kv=8, d=64, K=128, w=8,
         G=2, R=8, maxP=12, T=0, causal=True, is_cross=False, seed=21,
         store_inputs=False, grads=False),
]

CASE_BY_NAME = {c.name: c for c in CASES}
