"""Generate the golden fixtures by running the reference implementation.

Run where a checkout of the reference project is present (GPU boxes have
none), pointing at it with --ref or the SSA_REFERENCE environment variable:

    python tests/golden/make_golden.py --ref <reference checkout>

It imports the reference module unmodified and applies the two harness
canonicalisations the parity contract uses:

1. Stable bucket sort. The bucket sort at sparse_attention.py:781 calls
   `torch.sort` without `stable=True`; on CPU that order is not the ascending
   key order within a bucket. The harness forces `stable=True` for the duration
   of each call, which gives "ascending key index within a bucket", the order a
   counting sort produces. Outputs of the unpatched reference are recorded too
   (as a count of differing rows) so the difference stays visible.
2. fp32 hyperplanes. `rand_proj` stays fp32 while q/k/v are bf16; q/k/v are fed
   straight to `build_graph` / `apply_graph`, so the module is never cast.

For every case in cases.py it stores, as .npz: the per-round key/query bucket
ids, the LSH selection `lsh_idx`, the merged `neighbors`/`valid`, the attention
output and (when requested) the gradients of sum(out * dO) with respect to q,
k and v (k/v unexpanded: the GQA repeat is inside the autograd graph).
bf16 tensors are stored as their raw uint16 bit patterns.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from cases import CASES, derived, glob_list, make_inputs, checksum  # noqa: E402


@contextlib.contextmanager
def stable_sort():
    orig = torch.sort

    def _sort(*a, **kw):
        kw["stable"] = True
        return orig(*a, **kw)

    torch.sort = _sort
    try:
        yield
    finally:
        torch.sort = orig


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.bool:
        return t.numpy().astype(np.uint8)
    if t.dtype == torch.int64:
        return t.numpy().astype(np.int32)
    return t.numpy()


def small_idx(a: np.ndarray) -> np.ndarray:
    """Index arrays are stored in 16 bits when they fit (all cases here)."""
    if a.size == 0 or (a.min() >= 0 and a.max() < 32768):
        return a.astype(np.int16)
    return a.astype(np.int32)


def run_case(sa, c):
    dv = derived(c)
    q, k, v, rp, dO = make_inputs(c)
    rep = c.H // c.n_kv
    cfg = sa.SSAConfig(
        d_model=c.H * c.d, num_heads=c.H, num_kv_heads=c.n_kv,
        num_neighbors=c.K, max_num_hashes=c.maxP, num_hash_rounds=c.R,
        lsh_num_probes=c.T, window_size=c.w, num_global_tokens=c.G,
        global_token_indices=c.glob_idx, dropout=0.0, causal=c.causal,
        fp32_attn_weights=c.fp32_attn_weights)
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        attn = sa.SparseAttention(cfg)
    attn.eval()
    assert attn.lsh_k == dv["lsh_k"], (attn.lsh_k, dv)
    assert attn.lsh_builder.C == dv["C"]
    with torch.no_grad():
        attn.lsh_builder.rand_proj.copy_(rp)
    k_exp = k.repeat_interleave(rep, dim=1) if rep > 1 else k
    v_exp = v.repeat_interleave(rep, dim=1) if rep > 1 else v
    B, N, M = c.B, c.N, c.M
    causal = c.causal and not c.is_cross
    out = {}
    lsh = attn.lsh_builder
    p_eff = lsh.compute_effective_p(M, lsh.C, lsh.max_P)
    assert p_eff == dv["p_eff"], (p_eff, dv)
    with torch.no_grad(), stable_sort():
        glob = attn.glob_builder(M, "cpu")
        assert glob.tolist() == glob_list(c), (glob.tolist(), glob_list(c))
        # Per-round hash ids (sparse_attention.py:775-779).
        BH = B * c.H
        qf = q.reshape(BH, N, c.d)
        kf = k_exp.reshape(BH, M, c.d)
        kids, qids = [], []
        for r in range(c.R):
            kids.append(lsh._hash(kf, r, p_eff))
            qp = lsh._hash_proj(qf, r, p_eff)
            pw = 2 ** torch.arange(p_eff)
            qids.append(((qp > 0).long() * pw).sum(-1))
        out["k_ids"] = small_idx(torch.stack(kids, 1).numpy())   # (BH,R,M)
        out["q_ids"] = small_idx(torch.stack(qids, 1).numpy())   # (BH,R,N)
        lsh_idx = lsh(q, k_exp, attn.lsh_k, causal, glob)
        nb, valid = attn.build_graph(q, k_exp, N, M, B, "cpu", causal, c.is_cross)
        if c.store_inputs:
            out["lsh_idx"] = small_idx(to_np(lsh_idx))
            out["neighbors"] = small_idx(to_np(nb))
        else:
            # Large case: neighbor rows are ascending after slot 0, so a delta
            # encoding along the last axis compresses well; decode with cumsum.
            out["neighbors_delta"] = np.diff(to_np(nb), axis=-1, prepend=0).astype(np.int16)
            out["k_ids"] = out["k_ids"][:1]
            out["q_ids"] = out["q_ids"][:1]
        out["valid"] = np.packbits(to_np(valid), axis=-1) if not c.store_inputs else to_np(valid)
        o = attn.apply_graph(q, k_exp, v_exp, nb, valid)
        if c.store_inputs:
            out["out"] = to_np(o)
        else:
            out["out_checksum"] = np.array(checksum(o))
            out["out_rows"] = to_np(o.reshape(-1, c.d)[::997])
    # Unpatched (unstable sort) reference: count rows whose neighbor set differs.
    with torch.no_grad():
        nb_u, valid_u = attn.build_graph(q, k_exp, N, M, B, "cpu", causal, c.is_cross)
    same = ((nb_u == nb) | ~(valid_u | valid)).all(-1) & (valid_u == valid).all(-1)
    out["unstable_rows_differ"] = np.array(int((~same).sum()), dtype=np.int64)
    if c.grads:
        ql = q.clone().requires_grad_(True)
        kl = k.clone().requires_grad_(True)
        vl = v.clone().requires_grad_(True)
        ke = kl.repeat_interleave(rep, dim=1) if rep > 1 else kl
        ve = vl.repeat_interleave(rep, dim=1) if rep > 1 else vl
        o2 = attn.apply_graph(ql, ke, ve, nb, valid)
        (o2.float() * dO).sum().backward()
        out["dq"] = to_np(ql.grad)
        out["dk"] = to_np(kl.grad)
        out["dv"] = to_np(vl.grad)
    if c.store_inputs:
        out["q"], out["k"], out["v"] = to_np(q), to_np(k), to_np(v)
        out["rand_proj"] = rp.numpy()
        out["dO"] = dO.numpy()
    out["input_checksum"] = np.array(checksum(q) + checksum(k) + checksum(v) + checksum(rp))
    out["case_json"] = np.array(json.dumps(c.to_dict()))
    out["derived_json"] = np.array(json.dumps(dv))
    return out


def module_init_fixture(sa):
    """Weights of freshly constructed reference modules after manual_seed, so
    the new modules can be checked to consume the RNG in the same order."""
    res = {}
    torch.manual_seed(1234)
    cfg = sa.SSAConfig(d_model=32, num_heads=2, num_kv_heads=1, num_neighbors=12,
                       max_num_hashes=3, window_size=2, num_global_tokens=1)
    m = sa.SparseAttention(cfg)
    for kname, t in m.state_dict().items():
        res["attn." + kname] = t.numpy()
    torch.manual_seed(99)
    cfg2 = sa.SSAConfig(d_model=32, num_heads=2, num_neighbors=12,
                        max_num_hashes=2, window_size=3, num_global_tokens=1)
    tr = sa.SparseTransformer(cfg2, num_layers=2, vocab_size=50)
    for kname, t in tr.state_dict().items():
        res["tr." + kname] = t.numpy()
    torch.manual_seed(7)
    cg = sa.CachedGraphSparseTransformer(cfg2, num_layers=3, reuse_every=2)
    for kname, t in cg.state_dict().items():
        res["cg." + kname] = t.numpy()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SSA_REFERENCE"),
                    help="directory holding the reference's sparse_attention.py")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the reference checkout with --ref or SSA_REFERENCE")
    sys.path.insert(0, args.ref)
    import sparse_attention as sa  # the reference, unmodified
    torch.set_num_threads(os.cpu_count() or 1)
    meta = {"torch": torch.__version__, "cases": []}
    for c in CASES:
        if args.only and c.name != args.only:
            continue
        res = run_case(sa, c)
        np.savez_compressed(os.path.join(HERE, f"{c.name}.npz"), **res)
        meta["cases"].append({"name": c.name,
                              "unstable_rows_differ": int(res["unstable_rows_differ"])})
        print(c.name, "ok; unpatched-sort rows differing:", int(res["unstable_rows_differ"]))
    if not args.only:
        np.savez_compressed(os.path.join(HERE, "module_init.npz"), **module_init_fixture(sa))
        with open(os.path.join(HERE, "golden_meta.json"), "w") as f:
            json.dump(meta, f, indent=1)


if __name__ == "__main__":
    main()
