"""neighbor_overlap (sparse_attention.py:1583-1615) as a CUDA kernel, checked
against the reference's own broadcast formula restated in PyTorch, with
duplicates, padding and both index dtypes."""
import pytest
import torch

from ssa_b200 import ops
from ssa_b200.attention import SSAConfig, SparseTransformer, measure_cross_layer_overlap, neighbor_overlap

pytestmark = pytest.mark.gpu


def _formula(a, b, va, vb):
    a = torch.where(va, a, torch.full_like(a, -1))
    b = torch.where(vb, b, torch.full_like(b, -1))
    a_in_b = (a.unsqueeze(-1) == b.unsqueeze(-2)).any(dim=-1) & va
    inter = a_in_b.sum(dim=-1).float()
    union = (va.sum(dim=-1) + vb.sum(dim=-1)).float() - inter
    return inter / union.clamp_min(1.0)


@pytest.mark.parametrize("K,dtype", [(1, torch.int64), (7, torch.int32), (64, torch.int64), (129, torch.int32)])
def test_overlap_matches_reference_formula(cuda, K, dtype):
    g = torch.Generator(device="cpu").manual_seed(K)
    shape = (2, 3, 50, K)
    a = torch.randint(0, 3 * K + 1, shape, generator=g).to(dtype)   # duplicates happen
    b = torch.randint(0, 3 * K + 1, shape, generator=g).to(dtype)
    va = torch.rand(shape, generator=g) < 0.8
    vb = torch.rand(shape, generator=g) < 0.8
    va[0, 0, 0] = False                                             # an all-padding row
    vb[0, 0, 0] = False
    want = _formula(a, b, va, vb)
    got = neighbor_overlap(a.to(cuda), b.to(cuda), va.to(cuda), vb.to(cuda)).cpu()
    assert torch.equal(got, want)


def test_identical_graphs_overlap_one(cuda):
    nb = torch.arange(64, device=cuda).repeat(4, 1).view(1, 1, 4, 64)
    v = torch.ones_like(nb, dtype=torch.bool)
    assert torch.equal(ops.neighbor_overlap(nb, nb, v, v), torch.ones(1, 1, 4, device=cuda))


def test_measure_cross_layer_overlap_runs(cuda):
    cfg = SSAConfig(d_model=64, num_heads=2, num_neighbors=16, window_size=2, num_global_tokens=1,
                    num_hash_rounds=2, max_num_hashes=4, lsh_num_probes=0, dropout=0.0, causal=True)
    torch.manual_seed(0)
    model = SparseTransformer(cfg, num_layers=3, vocab_size=50).to(cuda).eval()
    x = torch.randint(0, 50, (2, 32), device=cuda)
    with torch.no_grad():
        stats = measure_cross_layer_overlap(model, x)
    assert stats["num_layers"] == 3 and len(stats["per_pair_overlap"]) == 2
    for ov in stats["mean_overlap_per_adjacent_pair"]:
        assert 0.0 <= ov <= 1.0
