"""Attention backward through the C ABI: the hand-written edge sort (the
inverted neighbor index) and its reuse across calls.

* Gradients against a plain PyTorch fp32 autograd reference of the
  reference's sparse_gather_attention (gather, fp32 softmax, weighted sum;
  sparse_attention.py:1096-1199) on graphs that exercise the sort: one, two
  and three 8-bit key digits (M < 256, M < 65536, M >= 65536), repeated
  indices within a row, out-of-range indices and invalid slots, GQA.
* ssa_attn_bwd_csr with an index built once (ssa_attn_build_csr) gives the
  same bits as ssa_attn_bwd, and a CachedGraphSparseTransformer group builds
  its index once for all of its layers.
"""
import numpy as np
import pytest
import torch

from ssa_b200 import _lib, ops
from ssa_b200.attention import CachedGraphSparseTransformer, SSAConfig

pytestmark = pytest.mark.gpu


def _torch_reference(q, k, v, nb, valid, scale):
    """fp32 autograd reference; k/v (B, n_kv, M, d) with head h reading kv
    head h // rep; slots that are invalid or out of [0, M) take no part."""
    B, H, N, d = q.shape
    n_kv, M = k.shape[1], k.shape[2]
    rep = H // n_kv
    kk = k.repeat_interleave(rep, dim=1)
    vv = v.repeat_interleave(rep, dim=1)
    ok = valid & (nb >= 0) & (nb < M)
    idx = torch.where(ok, nb, torch.zeros_like(nb)).long()
    bi = torch.arange(B).view(B, 1, 1, 1)
    hi = torch.arange(H).view(1, H, 1, 1)
    kg, vg = kk[bi, hi, idx], vv[bi, hi, idx]  # (B, H, N, Kn, d); backward accumulates into (B, H, M, d)
    s = torch.einsum("bhnd,bhnkd->bhnk", q, kg) * scale
    s = s.masked_fill(~ok, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bhnk,bhnkd->bhnd", p, vg)


@pytest.mark.parametrize("M,n_kv,H,dup", [(100, 2, 4, False), (300, 1, 4, True), (1030, 2, 2, True),
                                          (70000, 1, 2, False)])
def test_backward_matches_torch_autograd(cuda, M, n_kv, H, dup):
    g = torch.Generator().manual_seed(M)
    B, N, d, Kn = 2, 48, 32, 24
    q = torch.randn(B, H, N, d, generator=g)
    k = torch.randn(B, n_kv, M, d, generator=g)
    v = torch.randn(B, n_kv, M, d, generator=g)
    nb = torch.randint(0, M, (B, H, N, Kn), generator=g)
    if dup:  # repeated keys within a row, and indices outside [0, M)
        nb[..., 1] = nb[..., 0]
        nb[..., 2] = M + 5
        nb[..., 3] = -1
    valid = torch.rand(B, H, N, Kn, generator=g) > 0.2
    valid[..., 0] = True
    nb[..., 0] = nb[..., 0].clamp(0, M - 1)
    dO = torch.randn(B, H, N, d, generator=g)
    scale = d ** -0.5
    qr, kr, vr = (t.clone().requires_grad_() for t in (q, k, v))
    ref = _torch_reference(qr, kr, vr, nb, valid, scale)
    (ref * dO).sum().backward()
    qd, kd, vd = (t.to(cuda) for t in (q, k, v))
    nbd, vald = nb.to(cuda).int(), valid.to(cuda)
    out, lse = ops.attn_fwd(qd, kd, vd, nbd, vald, scale, False)
    assert torch.allclose(out.cpu(), ref.detach(), rtol=1e-4, atol=1e-5)
    dq, dk, dv = ops.attn_bwd(qd, kd, vd, nbd, vald, dO.to(cuda), lse, scale, False)
    for mine, r in ((dq, qr.grad), (dk, kr.grad), (dv, vr.grad)):
        err = (mine.cpu() - r).norm() / r.norm()
        assert err <= 1e-4, float(err)


def test_shared_index_gives_identical_gradients(cuda):
    g = torch.Generator().manual_seed(3)
    B, H, n_kv, N, M, d, Kn = 2, 8, 2, 256, 512, 64, 40
    q = torch.randn(B, H, N, d, generator=g).to(cuda, torch.bfloat16)
    k = torch.randn(B, n_kv, M, d, generator=g).to(cuda, torch.bfloat16)
    v = torch.randn(B, n_kv, M, d, generator=g).to(cuda, torch.bfloat16)
    nb = torch.randint(0, M, (B, H, N, Kn), generator=g).to(cuda).int()
    valid = (torch.rand(B, H, N, Kn, generator=g) > 0.1).to(cuda)
    out, lse = ops.attn_fwd(q, k, v, nb, valid, d ** -0.5, False)
    csr = ops.GraphCSR()
    for seed in range(3):  # three "layers" on one graph
        dO = torch.randn(B, H, N, d, generator=torch.Generator().manual_seed(seed)).to(cuda, torch.bfloat16)
        plain = ops.attn_bwd(q, k, v, nb, valid, dO, lse, d ** -0.5, False)
        shared = ops.attn_bwd(q, k, v, nb, valid, dO, lse, d ** -0.5, False, csr=csr)
        if seed == 0:
            buf = csr.buf
        assert csr.buf is buf, "the index was rebuilt for the same graph"
        for a, b in zip(plain, shared):
            assert torch.equal(a, b)


def test_cached_transformer_builds_one_index_per_group(cuda, monkeypatch):
    cfg = SSAConfig(d_model=64, num_heads=4, num_neighbors=32, window_size=2, num_global_tokens=1,
                    num_hash_rounds=2, max_num_hashes=4, causal=True)
    torch.manual_seed(0)
    model = CachedGraphSparseTransformer(cfg, num_layers=5, reuse_every=3).to(cuda)
    x = torch.randn(2, 64, 64, device=cuda, requires_grad=True)
    builds = []
    L = _lib.load()
    real = L.ssa_attn_build_csr

    class Counting:
        def __getattr__(self, name):
            return getattr(L, name)

        def ssa_attn_build_csr(self, *a):
            builds.append(1)
            return real(*a)

    monkeypatch.setattr(ops._lib, "load", lambda: Counting())
    out, _ = model(x)
    out.sum().backward()
    assert len(builds) == 2, builds  # groups {0, 1, 2} and {3, 4}
    assert torch.isfinite(x.grad).all()
    for layer in model.layers:
        assert layer.attn.Wq.weight.grad is not None and torch.isfinite(layer.attn.Wq.weight.grad).all()
