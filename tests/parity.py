"""Parity helpers shared by the GPU tests and smoke().

`compare_graphs` checks two neighbor graphs row by row. Rows must agree
exactly, except where the disagreement is explained by one of the two
causes the parity contract allows:

  * rescore tie -- every key in the symmetric difference of the two rows
    scores (exactly, in float64) within the fp32 rounding bound of a d-term
    dot product of the other swapped keys, i.e. the two selections differ
    only by the order of keys whose fp32 scores are indistinguishable;
  * hash near zero -- the query or a swapped key has a hyperplane
    projection within 1e-6 of zero in some round (checked by the caller
    through `hash_near_zero`).

It returns counts so the tests can assert "no unexplained row" and report
how many rows were explained by ties. `record` collects those counts per
case; when the environment variable SSA_PARITY_COUNTS names a file, the
test session writes them there as JSON (tests/conftest.py).
"""
from __future__ import annotations

import numpy as np

COUNTS: dict = {}


def record(case: str, **counts):
    """Adds per-case parity counts (rows compared, mismatched, ties, near-zero
    hash projections, unexplained) to the session's report."""
    entry = COUNTS.setdefault(case, {})
    for k, v in counts.items():
        entry[k] = int(v) if isinstance(v, (bool, int, np.integer)) else v


def rows_equal(nb_a, va_a, nb_b, va_b):
    """Per-row equality of (neighbors, valid), padding values ignored."""
    same_valid = (va_a == va_b).all(-1)
    same_nb = ((nb_a == nb_b) | ~va_a).all(-1)
    return same_valid & same_nb


def row_sets(nb, va):
    return set(nb[va].tolist())


def compare_graphs(nb_a, va_a, nb_b, va_b, q, k, n_kv, rel_tol=64.0 * 2.0 ** -24):
    """Compare graph a (e.g. GPU) against graph b (oracle / reference).

    nb_*/va_*: (B,H,N,W) int / bool numpy arrays. q (B,H,N,d), k
    (B,n_kv,M,d) float32. Returns dict(rows, mismatched, ties, unexplained,
    examples)."""
    B, H, N, W = nb_b.shape
    if nb_a.shape != nb_b.shape:
        return {"rows": B * H * N, "mismatched": B * H * N, "ties": 0,
                "unexplained": B * H * N, "examples": ["shape mismatch"]}
    eq = rows_equal(nb_a, va_a, nb_b, va_b)
    bad = np.argwhere(~eq)
    rep = H // n_kv
    ties, unexplained, examples = 0, 0, []
    for (b, h, n) in bad:
        sa = row_sets(nb_a[b, h, n], va_a[b, h, n])
        sb = row_sets(nb_b[b, h, n], va_b[b, h, n])
        diff = sorted(sa ^ sb)
        qv = q[b, h, n].astype(np.float64)
        kk = k[b, h // rep].astype(np.float64)
        sc = kk[diff] @ qv
        bound = rel_tol * (np.abs(kk[diff]) @ np.abs(qv)).max()
        if len(diff) and (sc.max() - sc.min()) <= 2 * bound:
            ties += 1
        else:
            unexplained += 1
            if len(examples) < 5:
                examples.append({"row": (int(b), int(h), int(n)), "only_a": sorted(sa - sb)[:8],
                                 "only_b": sorted(sb - sa)[:8],
                                 "scores": [float(x) for x in sc[:8]]})
    return {"rows": B * H * N, "mismatched": int(len(bad)), "ties": ties,
            "unexplained": unexplained, "examples": examples}


def hash_near_zero(x, rand_proj, p_eff, tol=1e-6):
    """(rows,) bool: some round's projection of the row is within tol of 0."""
    R = rand_proj.shape[0]
    planes = rand_proj[:, :p_eff].reshape(R * p_eff, -1).astype(np.float64)
    proj = x.reshape(-1, x.shape[-1]).astype(np.float64) @ planes.T
    return (np.abs(proj) < tol).any(-1)


def max_rel(a, b):
    """max |a - b| / max(|b|, tiny): the elementwise tolerance measure."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def norm_rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
