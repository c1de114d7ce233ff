"""Loader for the golden fixtures written by make_golden.py.

`load(name)` returns a dict with the case, its derived values, the inputs
(stored, or regenerated from the seed and checked against the stored
checksum) widened to float32 numpy arrays, and the reference outputs decoded
back to plain arrays (int32 indices, bool masks, float32 values).
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)

from cases import CASES, CASE_BY_NAME, Case, make_inputs, checksum, glob_list, derived  # noqa: E402,F401


def _widen(a: np.ndarray) -> np.ndarray:
    if a.dtype == np.uint16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a


def load(name: str) -> dict:
    c = CASE_BY_NAME[name]
    z = np.load(os.path.join(HERE, f"{name}.npz"))
    f = {k: z[k] for k in z.files}
    out = {"case": c, "derived": json.loads(str(f["derived_json"])), "glob": glob_list(c)}
    if c.store_inputs:
        out["q"], out["k"], out["v"] = (_widen(f["q"]), _widen(f["k"]), _widen(f["v"]))
        out["rand_proj"], out["dO"] = f["rand_proj"], f["dO"]
    else:
        q, k, v, rp, dO = make_inputs(c)
        cs = checksum(q) + checksum(k) + checksum(v) + checksum(rp)
        if not np.allclose(np.array(cs), f["input_checksum"], rtol=1e-12, atol=0):
            raise RuntimeError(f"regenerated inputs for {name} do not match the fixture")
        out["q"], out["k"], out["v"] = (q.float().numpy(), k.float().numpy(), v.float().numpy())
        out["rand_proj"], out["dO"] = rp.numpy(), dO.numpy()
    if "neighbors" in f:
        out["neighbors"] = f["neighbors"].astype(np.int32)
        out["valid"] = f["valid"].astype(bool)
    else:
        out["neighbors"] = np.cumsum(f["neighbors_delta"].astype(np.int32), axis=-1).astype(np.int32)
        Kout = out["neighbors"].shape[-1]
        out["valid"] = np.unpackbits(f["valid"], axis=-1)[..., :Kout].astype(bool)
    if "lsh_idx" in f:
        out["lsh_idx"] = f["lsh_idx"].astype(np.int32)
    out["k_ids"] = f["k_ids"].astype(np.int32)
    out["q_ids"] = f["q_ids"].astype(np.int32)
    for key in ("out", "dq", "dk", "dv"):
        if key in f:
            out[key] = _widen(f[key]).astype(np.float32)
    if "out_checksum" in f:
        out["out_checksum"] = f["out_checksum"]
        out["out_rows"] = _widen(f["out_rows"]).astype(np.float32)
    out["unstable_rows_differ"] = int(f["unstable_rows_differ"])
    return out
