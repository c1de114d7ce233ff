"""Attention-weight dropout (F.dropout after the weights' cast,
sparse_attention.py:1193-1194) on the GPU.

The keep decisions come from Philox4x32-10 inside the kernels; the tests
rebuild the same mask with the numpy restatement (tests/philox.py, pinned to
the generator's known-answer vectors), apply it in a plain PyTorch fp32
reference of the op and compare outputs and gradients. The reference's own
dropout tests (tests/test_review_coverage_gaps.py:133-188 there) only check
that training-mode outputs vary and that eval / p = 0 are deterministic;
those are ported below.
"""
import numpy as np
import pytest
import torch

from philox import dropout_keep
from ssa_b200 import ops
from ssa_b200.attention import SSAConfig, SparseAttention

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def _problem(dev, dtype, B=2, H=4, n_kv=2, N=96, M=128, d=64, Kn=40, seed=5):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, H, N, d, generator=g).to(device=dev, dtype=dtype)
    k = torch.randn(B, n_kv, M, d, generator=g).to(device=dev, dtype=dtype)
    v = torch.randn(B, n_kv, M, d, generator=g).to(device=dev, dtype=dtype)
    nb = torch.randint(0, M, (B, H, N, Kn), generator=g, dtype=torch.int32).to(dev)
    valid = torch.rand(B, H, N, Kn, generator=g) < 0.85
    valid[..., 0] = True
    return q, k, v, nb, valid.to(dev)


def _reference(q, k, v, nb, valid, scale, keep, p, fp32w):
    """PyTorch fp32 restatement of sparse_gather_attention with a given keep
    mask: returns (out, attn weights after dropout)."""
    B, H, N, d = q.shape
    rep = H // k.shape[1]
    kx = k.float().repeat_interleave(rep, 1)
    vx = v.float().repeat_interleave(rep, 1)
    idx = nb.long()
    kg = torch.gather(kx.unsqueeze(2).expand(B, H, N, *kx.shape[2:]), 3,
                      idx.unsqueeze(-1).expand(*idx.shape, d))
    vg = torch.gather(vx.unsqueeze(2).expand(B, H, N, *vx.shape[2:]), 3,
                      idx.unsqueeze(-1).expand(*idx.shape, d))
    s = torch.einsum("bhnd,bhnkd->bhnk", q.float(), kg) * scale
    s = s.masked_fill(~valid, float("-inf"))
    a = torch.softmax(s, dim=-1)
    if q.dtype == torch.bfloat16 and not fp32w:
        a = a.to(torch.bfloat16).float()
    scale_d = torch.tensor(1.0 / (1.0 - p), dtype=torch.float32)
    a = torch.where(keep, a * scale_d, torch.zeros_like(a))
    if q.dtype == torch.bfloat16 and not fp32w:
        a = a.to(torch.bfloat16).float()
    return torch.einsum("bhnk,bhnkd->bhnd", a, vg), a


def _keep_mask(shape, p, seed, offset=0):
    n = int(np.prod(shape))
    return torch.from_numpy(dropout_keep(np.arange(n, dtype=np.uint64), p, seed, offset).reshape(shape))


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


CASES = [(torch.bfloat16, 64, False), (torch.bfloat16, 32, False), (torch.float32, 64, False),
         (torch.bfloat16, 64, True)]


@pytest.mark.parametrize("dtype,d,fp32w", CASES)
def test_dropout_forward_matches_masked_reference(cuda, dtype, d, fp32w):
    p, seed = 0.3, 0x1234_5678_9ABC
    q, k, v, nb, valid = _problem(cuda, dtype, d=d)
    scale = d ** -0.5
    out, _ = ops.attn_fwd(q, k, v, nb, valid, scale, fp32w, want_lse=False, dropout=(p, seed, 0))
    keep = _keep_mask(nb.shape, p, seed).to(cuda)
    ref, _ = _reference(q, k, v, nb, valid, scale, keep, p, fp32w)
    assert _rel(out, ref) <= TOL[dtype]
    assert 0.6 < keep[valid].float().mean().item() < 0.8


@pytest.mark.parametrize("dtype,d,fp32w", CASES[:3])
def test_dropout_gradients_match_masked_reference(cuda, dtype, d, fp32w):
    p, seed = 0.25, 987654321
    q, k, v, nb, valid = _problem(cuda, dtype, d=d, seed=6)
    scale = d ** -0.5
    g = torch.Generator(device="cpu").manual_seed(11)
    dO = torch.randn(q.shape, generator=g).to(device=cuda, dtype=dtype)
    drop = (p, seed, 0)
    out, lse = ops.attn_fwd(q, k, v, nb, valid, scale, fp32w, dropout=drop)
    dq, dk, dv = ops.attn_bwd(q, k, v, nb, valid, dO, lse, scale, fp32w, dropout=drop)
    keep = _keep_mask(nb.shape, p, seed).to(cuda)
    with torch.no_grad():
        ref, _ = _reference(q, k, v, nb, valid, scale, keep, p, fp32w)
    # the fp32 reference differentiates through fp32 copies of q, k, v
    qr2, kr2, vr2 = (t.detach().float().requires_grad_() for t in (q, k, v))
    B, H, N, dd = qr2.shape
    rep = H // kr2.shape[1]
    kx, vx = kr2.repeat_interleave(rep, 1), vr2.repeat_interleave(rep, 1)
    idx = nb.long()
    kg = torch.gather(kx.unsqueeze(2).expand(B, H, N, *kx.shape[2:]), 3, idx.unsqueeze(-1).expand(*idx.shape, dd))
    vg = torch.gather(vx.unsqueeze(2).expand(B, H, N, *vx.shape[2:]), 3, idx.unsqueeze(-1).expand(*idx.shape, dd))
    s = (torch.einsum("bhnd,bhnkd->bhnk", qr2, kg) * scale).masked_fill(~valid, float("-inf"))
    a = torch.softmax(s, dim=-1) * keep * (1.0 / (1.0 - p))
    (torch.einsum("bhnk,bhnkd->bhnd", a, vg) * dO.float()).sum().backward()
    assert _rel(dq, qr2.grad) <= TOL[dtype]
    assert _rel(dk, kr2.grad) <= TOL[dtype]
    assert _rel(dv, vr2.grad) <= TOL[dtype]
    assert _rel(out, ref) <= TOL[dtype]


def _module(cuda, p):
    cfg = SSAConfig(d_model=128, num_heads=4, num_neighbors=32, window_size=4, num_global_tokens=2,
                    num_hash_rounds=2, max_num_hashes=6, lsh_num_probes=0, dropout=p, causal=False)
    torch.manual_seed(0)
    return SparseAttention(cfg).to(cuda)


def test_dropout_active_in_training_mode_changes_output(cuda):
    m = _module(cuda, 0.5).train()
    x = torch.randn(2, 64, 128, device=cuda)
    with torch.no_grad():
        a, _ = m(x)
        b, _ = m(x)
    assert not torch.allclose(a, b), "dropout=0.5 in training mode produced identical outputs across calls"


def test_dropout_inactive_in_eval_mode_is_deterministic(cuda):
    m = _module(cuda, 0.5).eval()
    x = torch.randn(2, 64, 128, device=cuda)
    with torch.no_grad():
        a, _ = m(x)
        b, _ = m(x)
    assert torch.equal(a, b)


def test_dropout_zero_is_deterministic_even_in_training_mode(cuda):
    m = _module(cuda, 0.0).train()
    x = torch.randn(2, 64, 128, device=cuda)
    with torch.no_grad():
        a, _ = m(x)
        b, _ = m(x)
    assert torch.equal(a, b)


def test_dropout_mask_follows_torch_seed_and_trains(cuda):
    m = _module(cuda, 0.2).train()
    x = torch.randn(2, 64, 128, device=cuda)
    torch.manual_seed(123)
    a, _ = m(x)
    torch.manual_seed(123)
    b, _ = m(x)
    assert torch.equal(a, b), "the same torch seed must give the same dropout mask"
    a.sum().backward()
    for name in ("Wq", "Wk", "Wv", "Wo"):
        w = getattr(m, name).weight
        assert w.grad is not None and torch.isfinite(w.grad).all(), name
