"""CUDA path vs the reference (golden fixtures) and vs the oracle.

Every golden case runs through the C ABI (ssa_b200.ops -> libssa_b200.so):
  * hash ids: bit-exact, except projections within 1e-6 of zero;
  * LSH selection (ssa_lsh_select): the reference's order, except ties;
  * merged graph (ssa_build_graph): neighbor lists and valid masks
    bit-exact; any differing row must be explained by a rescore tie;
  * gather attention forward on the reference graph: fp32 within 1e-4,
    bf16 within 2e-2 (relative to the largest output);
  * backward: dq, dk, dv within 1e-4 (fp32) / 2e-2 (bf16), norm-relative.
"""
import numpy as np
import pytest
import torch

from fixtures import CASES, load
from oracle import oracle as O
from parity import compare_graphs, hash_near_zero, max_rel, norm_rel, record

from ssa_b200 import ops

pytestmark = pytest.mark.gpu
NAMES = [c.name for c in CASES]


def _dev(a, dtype, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dtype)


def _inputs(g, dev):
    c = g["case"]
    dt = torch.float32 if c.dtype == "fp32" else torch.bfloat16
    q = _dev(g["q"], dt, dev)
    k = _dev(g["k"], dt, dev)
    v = _dev(g["v"], dt, dev)
    rp = _dev(g["rand_proj"], torch.float32, dev)
    glob = torch.tensor(g["glob"], dtype=torch.int32, device=dev)
    return q, k, v, rp, glob


@pytest.mark.parametrize("name", NAMES)
def test_hash_ids_match_reference(name, cuda):
    g = load(name)
    c, dv = g["case"], g["derived"]
    q, k, v, rp, glob = _inputs(g, cuda)
    kid = ops.hash_ids(k, rp, c.R, c.maxP, dv["p_eff"]).cpu().numpy()       # (B*n_kv, R, M)
    qid = ops.hash_ids(q, rp, c.R, c.maxP, dv["p_eff"]).cpu().numpy()       # (B*H, R, N)
    rep = c.H // c.n_kv
    bh = np.arange(c.B * c.H)
    kid_exp = kid[(bh // c.H) * c.n_kv + (bh % c.H) // rep]
    nref = g["k_ids"].shape[0]
    kbad = kid_exp[:nref] != g["k_ids"]
    qbad = qid[:nref] != g["q_ids"]
    record(name, hash_ids_compared=kbad.size + qbad.size, hash_ids_mismatched=kbad.sum() + qbad.sum())
    if kbad.any():
        rows = np.unique(np.argwhere(kbad)[:, [0, 2]], axis=0)
        kk = g["k"].reshape(c.B * c.n_kv, c.M, c.d)
        for bh_i, m in rows:
            bgi = (bh_i // c.H) * c.n_kv + (bh_i % c.H) // rep
            assert hash_near_zero(kk[bgi, m][None], g["rand_proj"], dv["p_eff"])[0]
    if qbad.any():
        rows = np.unique(np.argwhere(qbad)[:, [0, 2]], axis=0)
        qq = g["q"].reshape(c.B * c.H, c.N, c.d)
        for bh_i, n in rows:
            assert hash_near_zero(qq[bh_i, n][None], g["rand_proj"], dv["p_eff"])[0]


@pytest.mark.parametrize("name", NAMES)
def test_graph_matches_reference(name, cuda):
    g = load(name)
    c, dv = g["case"], g["derived"]
    q, k, v, rp, glob = _inputs(g, cuda)
    nb, valid = ops.build_graph(q, k, rp, glob, R=c.R, max_p=c.maxP, p_eff=dv["p_eff"], C=dv["C"],
                                T=c.T, A=dv["A"], causal=c.causal and not c.is_cross,
                                is_cross=c.is_cross, K=c.K, window=c.w)
    torch.cuda.synchronize()
    res = compare_graphs(nb.cpu().numpy(), valid.cpu().numpy().astype(bool), g["neighbors"],
                         g["valid"], g["q"], g["k"], c.n_kv)
    print(name, {k_: res[k_] for k_ in ("rows", "mismatched", "ties")})
    record(name, graph_rows=res["rows"], graph_mismatched=res["mismatched"], graph_ties=res["ties"],
           graph_unexplained=res["unexplained"])
    assert res["unexplained"] == 0, res
    assert res["ties"] <= max(2, res["rows"] // 1000), res


@pytest.mark.parametrize("name", [n for n in NAMES if n != "c1_full"])
def test_lsh_select_matches_reference_order(name, cuda):
    g = load(name)
    c, dv = g["case"], g["derived"]
    q, k, v, rp, glob = _inputs(g, cuda)
    out = ops.lsh_select(q, k, rp, glob, R=c.R, max_p=c.maxP, p_eff=dv["p_eff"], C=dv["C"], T=c.T,
                         A=dv["A"], causal=c.causal and not c.is_cross).cpu().numpy()
    ref = g["lsh_idx"]
    same_set = (np.sort(out, -1) == np.sort(ref, -1)).all(-1)
    if name == "zero_keys_fallback":  # every score is exactly 0: only the set is defined
        assert same_set.all()
        return
    differ = ~(out == ref).all(-1)
    record(name, lsh_order_rows=differ.size, lsh_order_differ=differ.sum())
    assert differ.sum() <= max(2, differ.size // 1000), int(differ.sum())


@pytest.mark.parametrize("name", NAMES)
def test_attention_forward_matches_reference(name, cuda):
    g = load(name)
    c = g["case"]
    q, k, v, rp, glob = _inputs(g, cuda)
    nb = torch.from_numpy(g["neighbors"]).to(cuda)
    va = torch.from_numpy(g["valid"]).to(cuda)
    out, lse = ops.attn_fwd(q, k, v, nb, va, c.d ** -0.5, c.fp32_attn_weights)
    out = out.float().cpu().numpy()
    lowp = c.dtype == "bf16"
    tol = 2e-2 if lowp else 1e-4
    ora, _ = O.attn_fwd(g["q"], g["k"], g["v"], g["neighbors"], g["valid"], scale=c.d ** -0.5,
                        lowp=lowp, fp32_w=c.fp32_attn_weights)
    assert max_rel(out, ora) <= tol
    if "out" in g:
        assert max_rel(out, g["out"]) <= tol
    # int64 neighbors + bool valid (the reference's dtypes) give the same result
    out64, _ = ops.attn_fwd(q, k, v, nb.long(), va.bool(), c.d ** -0.5, c.fp32_attn_weights)
    assert torch.equal(out64.float().cpu(), torch.from_numpy(out))


@pytest.mark.parametrize("name", [c.name for c in CASES if c.grads])
def test_attention_backward_matches_reference(name, cuda):
    g = load(name)
    c = g["case"]
    q, k, v, rp, glob = _inputs(g, cuda)
    nb = torch.from_numpy(g["neighbors"]).to(cuda)
    va = torch.from_numpy(g["valid"]).to(cuda)
    out, lse = ops.attn_fwd(q, k, v, nb, va, c.d ** -0.5, c.fp32_attn_weights)
    dO = _dev(g["dO"], q.dtype, cuda)
    dq, dk, dv = ops.attn_bwd(q, k, v, nb, va, dO, lse, c.d ** -0.5, c.fp32_attn_weights)
    lowp = c.dtype == "bf16"
    tol = 2e-2 if lowp else 1e-4
    oq, ok_, ov = O.attn_bwd(g["q"], g["k"], g["v"], g["neighbors"], g["valid"], g["dO"],
                             scale=c.d ** -0.5, lowp=lowp, fp32_w=c.fp32_attn_weights)
    for mine, ora, ref in ((dq, oq, g["dq"]), (dk, ok_, g["dk"]), (dv, ov, g["dv"])):
        m = mine.float().cpu().numpy()
        assert norm_rel(m, ora) <= tol
        assert norm_rel(m, ref) <= tol


def test_backward_is_deterministic(cuda):
    g = load("c2s_bf16_gqa_causal")
    c = g["case"]
    q, k, v, rp, glob = _inputs(g, cuda)
    nb = torch.from_numpy(g["neighbors"]).to(cuda)
    va = torch.from_numpy(g["valid"]).to(cuda)
    out, lse = ops.attn_fwd(q, k, v, nb, va, c.d ** -0.5, False)
    dO = _dev(g["dO"], q.dtype, cuda)
    r1 = ops.attn_bwd(q, k, v, nb, va, dO, lse, c.d ** -0.5, False)
    r2 = ops.attn_bwd(q, k, v, nb, va, dO, lse, c.d ** -0.5, False)
    for a, b in zip(r1, r2):
        assert torch.equal(a, b)
