"""The reference suite's invariants (tests/*.py of daedalus/SSA), re-stated
against the B200 modules on CUDA: shapes and the stats contract, dedup and
the self slot, the empty-bucket fallback, causal leakage, cross-attention
ranges, GQA/MQA, explicit globals, the build/apply split, gradients,
multi-probe, recall, the cached-graph transformer and fp32 weights."""
import pytest
import torch

from ssa_b200 import (
    CachedGraphSparseTransformer, GlobalGraphBuilder, LSHGraphBuilder, SSAConfig, SparseAttention,
    SparseTransformer, WindowGraphBuilder, merge_neighbors, neighbor_overlap,
    measure_cross_layer_overlap,
)

pytestmark = pytest.mark.gpu


@pytest.fixture
def base_cfg():
    return SSAConfig(d_model=128, num_heads=2, num_neighbors=32, max_num_hashes=3, window_size=4,
                     num_global_tokens=2, dropout=0.0, causal=False)


@pytest.fixture
def causal_cfg():
    return SSAConfig(d_model=64, num_heads=2, num_neighbors=16, max_num_hashes=2, window_size=3,
                     num_global_tokens=1, causal=True)


def test_self_attention_shapes_and_stats(base_cfg, cuda):
    model = SparseTransformer(base_cfg, num_layers=2).to(cuda)
    x = torch.randn(2, 64, base_cfg.d_model, device=cuda)
    out, stats = model(x, return_stats=True)
    assert out.shape == x.shape
    assert stats[0]["neighbors_shape"] == (2, base_cfg.num_heads, 64, base_cfg.num_neighbors)
    assert stats[0]["compression"] > 1.0
    out, stats = model(x)
    assert all(s == {} for s in stats)


def test_cross_attention_shape_and_range(base_cfg, cuda):
    attn = SparseAttention(base_cfg).to(cuda).eval()
    qx = torch.randn(1, 48, base_cfg.d_model, device=cuda)
    kv = torch.randn(1, 96, base_cfg.d_model, device=cuda)
    out, stats = attn(qx, key_value=kv, return_stats=True)
    assert out.shape == qx.shape
    assert stats["neighbors_shape"][:3] == (1, base_cfg.num_heads, 48)
    with torch.no_grad():
        q = attn._split_q(attn.Wq(qx))
        k = attn._split_kv(attn.Wk(kv))
        nb, valid = attn.build_graph(q, k, N=48, M=96, B=1, device=cuda, causal=False, is_cross=True)
    assert nb.dtype == torch.int64 and valid.dtype == torch.bool
    assert bool((nb[valid] < 96).all()) and bool((nb[valid] >= 0).all())


def test_merge_no_duplicates_and_self_first(cuda):
    win = WindowGraphBuilder(4)(32, 32, cuda)
    glob = GlobalGraphBuilder(2)(32, cuda)
    lsh = LSHGraphBuilder(d_head=8, lsh_candidates=8, num_rounds=2).to(cuda)
    q = torch.randn(1, 1, 32, 8, device=cuda)
    k = torch.randn(1, 1, 32, 8, device=cuda)
    lsh_idx = lsh(q, k, top_k=4)
    self_idx = torch.arange(32, device=cuda).view(1, 1, 32)
    nb, valid = merge_neighbors(win, glob, lsh_idx, self_idx=self_idx, total_k=24, N=32, B=1, H=1,
                                device=cuda)
    assert bool((nb[0, 0, :, 0] == torch.arange(32, device=cuda)).all())
    for i in range(32):
        slots = nb[0, 0, i, 1:][valid[0, 0, i, 1:]].tolist()
        assert len(slots) == len(set(slots))


def test_empty_bucket_fallback_uses_globals(cuda):
    lsh = LSHGraphBuilder(d_head=4, max_num_hashes=1, lsh_candidates=4).to(cuda)
    k = torch.zeros(1, 1, 8, 4, device=cuda)      # every key in bucket 0
    q = torch.ones(1, 1, 4, 4, device=cuda)
    lsh.rand_proj.copy_(lsh.rand_proj.abs())     # queries land in bucket 1 (empty)
    nb = lsh(q, k, top_k=2, causal=False, glob_fallback=torch.tensor([0, 1], device=cuda))
    assert not bool((nb == 7).all())
    assert set(nb[0, 0, 0].tolist()) <= {0, 1}


def test_cross_attention_more_queries_than_keys(cuda):
    cfg = SSAConfig(d_model=16, num_heads=1, num_neighbors=4, max_num_hashes=1, window_size=1,
                    num_global_tokens=1, causal=False)
    attn = SparseAttention(cfg).to(cuda)
    out, _ = attn(torch.randn(1, 10, 16, device=cuda), key_value=torch.randn(1, 3, 16, device=cuda))
    assert out.shape == (1, 10, 16) and not bool(out.isnan().any())


def test_causal_no_future_leak(causal_cfg, cuda):
    N = 32
    lsh = LSHGraphBuilder(d_head=8, max_num_hashes=2, lsh_candidates=8).to(cuda)
    q = torch.randn(1, 1, N, 8, device=cuda)
    k = torch.randn(1, 1, N, 8, device=cuda)
    nb = lsh(q, k, top_k=4, causal=True, glob_fallback=torch.zeros(1, dtype=torch.long, device=cuda))
    for i in range(N):
        assert not bool((nb[0, 0, i] > i).any())
    attn = SparseAttention(causal_cfg).to(cuda)
    out, _ = attn(torch.randn(1, 32, causal_cfg.d_model, device=cuda))
    assert not bool(out.isnan().any())


def test_causal_with_probes_no_leak(cuda):
    cfg = SSAConfig(d_model=32, num_heads=2, num_neighbors=32, max_num_hashes=6, num_hash_rounds=2,
                    window_size=2, num_global_tokens=1, causal=True, lsh_num_probes=3)
    attn = SparseAttention(cfg).to(cuda).eval()
    N = 200
    x = torch.randn(1, N, 32, device=cuda)
    with torch.no_grad():
        nb, valid = attn.build_graph(attn._split_q(attn.Wq(x)), attn._split_kv(attn.Wk(x)), N, N, 1,
                                     cuda, causal=True, is_cross=False)
    glob = {0}
    for i in range(N):
        idx = nb[0, 0, i][valid[0, 0, i]]
        assert all(j <= i or j in glob for j in idx.tolist())


def test_gqa_mqa_shapes_and_params(cuda):
    for n_kv in (1, 2, 4):
        cfg = SSAConfig(d_model=64, num_heads=4, num_kv_heads=n_kv, num_neighbors=16,
                        window_size=4, num_global_tokens=2, max_num_hashes=3)
        attn = SparseAttention(cfg).to(cuda)
        x = torch.randn(2, 32, 64, device=cuda, requires_grad=True)
        out, _ = attn(x)
        assert out.shape == x.shape
        out.sum().backward()
        assert not bool(x.grad.isnan().any())
        assert attn.Wk.weight.grad.norm().item() > 0
        assert attn.Wk.weight.numel() == 64 * 16 * n_kv
    with pytest.raises(AssertionError):
        SparseAttention(SSAConfig(d_model=64, num_heads=5, num_kv_heads=2))


def test_explicit_globals(cuda):
    cfg = SSAConfig(d_model=64, num_heads=2, num_neighbors=16, window_size=4, num_global_tokens=2,
                    global_token_indices=[0, 15, 31], max_num_hashes=3)
    attn = SparseAttention(cfg).to(cuda)
    out, _ = attn(torch.randn(2, 32, 64, device=cuda))
    assert out.shape == (2, 32, 64)
    assert GlobalGraphBuilder(2, [0, 5, 17])(32, cuda).tolist() == [0, 5, 17]
    assert GlobalGraphBuilder(2, [0, 100, 200])(32, cuda).max().item() <= 31


@pytest.mark.parametrize("kind", ["self", "cross", "causal"])
def test_build_apply_split_matches_forward(kind, base_cfg, causal_cfg, cuda):
    cfg = causal_cfg if kind == "causal" else base_cfg
    attn = SparseAttention(cfg).to(cuda).eval()
    x = torch.randn(2, 48, cfg.d_model, device=cuda)
    kv = torch.randn(2, 80, cfg.d_model, device=cuda) if kind == "cross" else None
    with torch.no_grad():
        direct, _ = attn(x, key_value=kv)
        src = kv if kv is not None else x
        q = attn._split_q(attn.Wq(x))
        k = attn._split_kv(attn.Wk(src))
        v = attn._split_kv(attn.Wv(src))
        nb, valid = attn.build_graph(q, k, N=48, M=src.shape[1], B=2, device=cuda,
                                     causal=cfg.causal, is_cross=kv is not None)
        split = attn.Wo(attn._merge(attn.apply_graph(q, k, v, nb, valid)))
    assert torch.allclose(direct, split, atol=1e-6)


def test_gradients_reach_every_projection(cuda):
    cfg = SSAConfig(d_model=32, num_heads=2, num_neighbors=12, max_num_hashes=2, window_size=3,
                    num_global_tokens=1)
    attn = SparseAttention(cfg).to(cuda)
    x = torch.randn(2, 24, 32, device=cuda, requires_grad=True)
    out, _ = attn(x)
    out.sum().backward()
    for lin in (attn.Wq, attn.Wk, attn.Wv, attn.Wo):
        assert lin.weight.grad is not None and lin.weight.grad.norm().item() > 0
    model = SparseTransformer(cfg, num_layers=2, vocab_size=50).to(cuda)
    ids = torch.randint(0, 50, (1, 16), device=cuda)
    out, _ = model(ids)
    out.sum().backward()
    assert model.embed.weight.grad is not None and not bool(model.embed.weight.grad.isnan().any())


def test_recall_beats_random(cuda):
    torch.manual_seed(0)
    N, d_model = 1024, 64
    cfg = SSAConfig(d_model=d_model, num_heads=2, num_neighbors=64, max_num_hashes=12,
                    num_hash_rounds=4, window_size=8, num_global_tokens=4, causal=False)
    attn = SparseAttention(cfg).to(cuda).eval()
    x = torch.randn(1, N, d_model, device=cuda)
    with torch.no_grad():
        q = attn._split_q(attn.Wq(x))
        k = attn._split_kv(attn.Wk(x))
        glob = attn.glob_builder(N, cuda)
        win = attn.win_builder(N, N, cuda)
        lsh_idx = attn.lsh_builder(q, k, attn.lsh_k, False, glob)
        self_idx = torch.arange(N, device=cuda).view(1, 1, N).expand(1, 2, N)
        nb, valid = merge_neighbors(win, glob, lsh_idx, self_idx, cfg.num_neighbors, N, 1, 2, cuda)
    true_top = (q[0, 0] @ k[0, 0].T).topk(32, dim=-1).indices
    hit = torch.zeros(N, device=cuda)
    for i in range(N):
        sparse = set(nb[0, 0, i][valid[0, 0, i]].tolist())
        hit[i] = len(sparse & set(true_top[i].tolist())) / 32
    rand_floor = cfg.num_neighbors / N
    assert hit.mean().item() > 2 * rand_floor


def test_recall_rises_with_probes(cuda):
    def recall(T):
        torch.manual_seed(0)
        cfg = SSAConfig(d_model=32, num_heads=2, num_neighbors=64, max_num_hashes=12,
                        num_hash_rounds=4, lsh_num_probes=T, window_size=8, num_global_tokens=4)
        attn = SparseAttention(cfg).to(cuda).eval()
        N = 2048
        x = torch.randn(1, N, 32, device=cuda)
        with torch.no_grad():
            q = attn._split_q(attn.Wq(x))
            k = attn._split_kv(attn.Wk(x))
            nb, valid = attn.build_graph(q, k, N, N, 1, cuda, False, False)
        top = (q[0, 0] @ k[0, 0].T).topk(32, dim=-1).indices
        member = torch.zeros(N, N, dtype=torch.bool, device=cuda)
        rows = torch.arange(N, device=cuda).unsqueeze(1).expand_as(nb[0, 0])
        member[rows[valid[0, 0]], nb[0, 0][valid[0, 0]]] = True
        return member.gather(1, top).float().mean().item()
    r0, r1, r3 = recall(0), recall(1), recall(3)
    assert r0 < r1 < r3


def test_cached_graph_transformer(base_cfg, cuda):
    model = CachedGraphSparseTransformer(base_cfg, num_layers=6, reuse_every=3).to(cuda)
    x = torch.randn(2, 48, base_cfg.d_model, device=cuda, requires_grad=True)
    out, stats = model(x, return_stats=True)
    assert out.shape == x.shape and len(stats) == 6
    assert [s["graph_recomputed"] for s in stats] == [True, False, False, True, False, False]
    out.sum().backward()
    assert not bool(x.grad.isnan().any()) and x.grad.norm().item() > 0


def test_overlap_diagnostics(base_cfg, cuda):
    idx = torch.randint(0, 16, (1, 2, 8, 4), device=cuda)
    ones = torch.ones_like(idx, dtype=torch.bool)
    assert torch.allclose(neighbor_overlap(idx, idx, ones, ones), torch.ones(1, 2, 8, device=cuda))
    model = SparseTransformer(base_cfg, num_layers=3).to(cuda)
    rep = measure_cross_layer_overlap(model, torch.randn(1, 32, base_cfg.d_model, device=cuda))
    assert len(rep["mean_overlap_per_adjacent_pair"]) == 2


def test_fp32_weights_close_to_default_in_fp32(cuda):
    base = dict(d_model=32, num_heads=2, num_neighbors=12, max_num_hashes=2, window_size=3,
                num_global_tokens=1)
    torch.manual_seed(123)
    a = SparseAttention(SSAConfig(**base, fp32_attn_weights=False)).to(cuda)
    torch.manual_seed(123)
    b = SparseAttention(SSAConfig(**base, fp32_attn_weights=True)).to(cuda)
    x = torch.randn(1, 24, 32, device=cuda)
    assert torch.allclose(a(x)[0], b(x)[0], atol=1e-5)


def test_bf16_module_keeps_fp32_hyperplanes(cuda):
    cfg = SSAConfig(d_model=256, num_heads=2, num_kv_heads=1, num_neighbors=32, window_size=2)
    attn = SparseAttention(cfg).to(cuda, torch.bfloat16)
    assert attn.lsh_builder.rand_proj.dtype == torch.float32
    out, _ = attn(torch.randn(1, 64, 256, device=cuda, dtype=torch.bfloat16))
    assert out.dtype == torch.bfloat16 and bool(torch.isfinite(out.float()).all())


def test_invalid_inputs_raise(cuda):
    attn = SparseAttention(SSAConfig(d_model=32, num_heads=2, num_neighbors=12, window_size=2)).to(cuda)
    with pytest.raises(ValueError, match="attention_mask"):
        attn(torch.randn(1, 8, 32, device=cuda), attention_mask=torch.ones(1, 8, device=cuda))
    half = attn.half()
    assert half.lsh_builder.rand_proj.dtype == torch.float32
    with pytest.raises(NotImplementedError):
        half(torch.randn(1, 8, 32, device=cuda, dtype=torch.float16))
