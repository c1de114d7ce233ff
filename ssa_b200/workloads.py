"""The five benchmark configurations of the reference's headline metric, as
seeded synthetic workloads.

No dataset is involved: inputs are drawn from seeded generators with the
shapes and distributions the configurations name (N(0, 1) activations; a
64-centre Gaussian mixture with sigma 0.3 for the long-context config;
uniform token ids for the training config). Module weights are random-init
in the reference's construction order (seed 0), inputs use seed 1.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .attention import SSAConfig, SparseAttention


@dataclass(frozen=True)
class Workload:
    name: str
    dtype: str
    B: int
    N: int
    M: int
    d_model: int
    H: int
    n_kv: int
    K: int
    window: int
    G: int
    glob: Optional[tuple]
    R: int
    max_p: int
    T: int
    causal: bool
    cross: bool
    inputs: str
    layers: int = 1
    vocab: int = 0

    @property
    def d(self) -> int:
        return self.d_model // self.H

    @property
    def torch_dtype(self):
        return torch.float32 if self.dtype == "fp32" else torch.bfloat16

    def config(self) -> SSAConfig:
        return SSAConfig(d_model=self.d_model, num_heads=self.H, num_kv_heads=self.n_kv,
                         num_neighbors=self.K, max_num_hashes=self.max_p, num_hash_rounds=self.R,
                         lsh_num_probes=self.T, window_size=self.window, num_global_tokens=self.G,
                         global_token_indices=list(self.glob) if self.glob else None,
                         dropout=0.0, causal=self.causal)

    def bytes_per_token(self) -> int:
        """Algorithmic bytes of gather attention per token (all heads):
        H * (2 K d s + 2 d s) -- the gathered K and V rows plus the q row
        read and the output row written."""
        s = 4 if self.dtype == "fp32" else 2
        return self.H * (2 * self.K * self.d * s + 2 * self.d * s)


WORKLOADS = {
    "c1": Workload("c1", "fp32", B=2, N=1024, M=1024, d_model=512, H=8, n_kv=8, K=128, window=8,
                   G=2, glob=None, R=8, max_p=12, T=0, causal=True, cross=False, inputs="normal"),
    "c2": Workload("c2", "bf16", B=4, N=8192, M=8192, d_model=4096, H=32, n_kv=8, K=128,
                   window=16, G=4, glob=None, R=8, max_p=12, T=0, causal=True, cross=False,
                   inputs="normal"),
    "c3": Workload("c3", "bf16", B=1, N=32768, M=32768, d_model=1024, H=16, n_kv=16, K=256,
                   window=32, G=4, glob=None, R=8, max_p=12, T=2, causal=False, cross=False,
                   inputs="cluster"),
    "c4": Workload("c4", "fp32", B=16, N=1024, M=1024, d_model=512, H=8, n_kv=8, K=128, window=8,
                   G=2, glob=None, R=8, max_p=12, T=0, causal=True, cross=False, inputs="tokens",
                   layers=6, vocab=32000),
    "c5": Workload("c5", "bf16", B=8, N=4096, M=8192, d_model=2048, H=32, n_kv=1, K=128, window=8,
                   G=0, glob=(0, 1, 4096), R=8, max_p=12, T=1, causal=False, cross=True,
                   inputs="normal"),
}


def make_module(w: Workload, device, seed: int = 0) -> SparseAttention:
    torch.manual_seed(seed)
    m = SparseAttention(w.config())
    return m.to(device=device, dtype=w.torch_dtype).eval()


def make_x(w: Workload, device, seed: int = 1, batch: Optional[int] = None, rows=None):
    """Activations (B, N, d_model) and, for cross-attention, the key/value
    source (B, M, d_model). `rows` (start, stop) draws only a slice of the
    sequence from the same stream (the generator is advanced exactly)."""
    B = batch if batch is not None else w.B
    g = torch.Generator(device="cpu").manual_seed(seed)
    if w.inputs == "cluster":
        cent = torch.randn(64, w.d_model, generator=g)
        assign = torch.randint(0, 64, (B, w.N), generator=g)
        x = cent[assign] + 0.3 * torch.randn(B, w.N, w.d_model, generator=g)
        kv = None
    else:
        x = torch.randn(B, w.N, w.d_model, generator=g)
        kv = torch.randn(B, w.M, w.d_model, generator=g) if w.cross else None
    x = x.to(device=device, dtype=w.torch_dtype)
    kv = kv.to(device=device, dtype=w.torch_dtype) if kv is not None else None
    return x, kv


@torch.no_grad()
def project(m: SparseAttention, x: torch.Tensor, kv: Optional[torch.Tensor] = None):
    """q (B,H,N,d) and unexpanded k, v (B,n_kv,M,d) as strided views of the
    projection outputs -- the layout the kernels consume directly."""
    src = kv if kv is not None else x
    return m._split_q(m.Wq(x)), m._split_kv_grouped(m.Wk(src)), m._split_kv_grouped(m.Wv(src))
