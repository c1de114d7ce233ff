"""Sharding on one GPU: the pieces a rank computes, checked against the
unsharded build of the same job. Size-independent properties; the row
offset (q_row0) and the group slices must reproduce the full graph's rows
and heads bit for bit, and the full attention output."""
import pytest
import torch

from ssa_b200 import ops
from ssa_b200.attention import SSAConfig, SparseAttention
from ssa_b200.sharding import GroupSharded, group_slices, slice_views, split_range

pytestmark = pytest.mark.gpu


def _setup(cuda, dtype, causal, H=8, n_kv=2, N=1024, d=64, K=64, w=4, T=1, B=2, clustered=False):
    cfg = SSAConfig(d_model=H * d, num_heads=H, num_kv_heads=n_kv, num_neighbors=K, window_size=w,
                    num_global_tokens=2, num_hash_rounds=4, max_num_hashes=8, lsh_num_probes=T,
                    dropout=0.0, causal=causal)
    torch.manual_seed(0)
    m = SparseAttention(cfg).to(device=cuda, dtype=dtype).eval()
    g = torch.Generator(device="cpu").manual_seed(1)
    if clustered:
        cent = torch.randn(16, H * d, generator=g)
        x = cent[torch.randint(0, 16, (B, N), generator=g)] + 0.3 * torch.randn(B, N, H * d, generator=g)
    else:
        x = torch.randn(B, N, H * d, generator=g)
    x = x.to(device=cuda, dtype=dtype)
    with torch.no_grad():
        q = m.Wq(x).view(B, N, H, d).transpose(1, 2)
        k = m.Wk(x).view(B, N, n_kv, d).transpose(1, 2)
        v = m.Wv(x).view(B, N, n_kv, d).transpose(1, 2)
    return m, q, k, v


CASES = [(torch.bfloat16, True, False), (torch.bfloat16, False, True), (torch.float32, True, False)]


@pytest.mark.parametrize("dtype,causal,clustered", CASES)
def test_row_slices_reproduce_full_graph(cuda, dtype, causal, clustered):
    m, q, k, v = _setup(cuda, dtype, causal, clustered=clustered)
    N = q.shape[2]
    with torch.no_grad():
        nb, valid = m._graph(q, k, N, causal, False)
        for world in (2, 4, 3):
            for rank in range(world):
                r0, r1 = split_range(N, world, rank)
                nbs, vs = m._graph(q[:, :, r0:r1], k, N, causal, False, q_row0=r0)
                assert torch.equal(nbs, nb[:, :, r0:r1]), f"neighbors differ, world {world} rank {rank}"
                assert torch.equal(vs, valid[:, :, r0:r1]), f"valid differs, world {world} rank {rank}"


@pytest.mark.parametrize("dtype,causal,clustered", CASES[:2])
def test_group_shards_reproduce_full_attention(cuda, dtype, causal, clustered):
    m, q, k, v = _setup(cuda, dtype, causal, clustered=clustered)
    B, H, N, d = q.shape
    n_kv = k.shape[1]
    rep = H // n_kv
    with torch.no_grad():
        nb, valid = m._graph(q, k, N, causal, False)
        ref, _ = ops.attn_fwd(q, k, v, nb, valid, m.scale, False, want_lse=False)
        for world in (2, 3, 4):
            out = torch.full_like(ref, float("nan"))
            for rank in range(world):
                for s, o in GroupSharded(m, world, rank, causal=causal).step(q, k, v):
                    out[s.b0:s.b1, s.g0 * rep:s.g1 * rep] = o
            assert torch.equal(out, ref), f"world {world}"
    assert sum(len(group_slices(B, n_kv, 4, r)) for r in range(4)) >= 4
    qs, ks, vs = slice_views(q, k, v, group_slices(B, n_kv, 4, 1)[0], rep)
    assert qs.shape[1] == rep * ks.shape[1]
