"""Failure path of the tensor-core candidate scan, without a GPU fault.

Every wait of the scan on an on-chip barrier is bounded. Here the bound is
cut to one poll (ssa_debug_set_wait_limit), so waits run out on a real
build: the kernels must return, ssa_device_error must report one of the
scan's wait codes, and the next build with the default bound must give
exactly the graph of a clean build -- the context stays usable.
"""
import numpy as np
import pytest
import torch

from fixtures import load

from ssa_b200 import _lib, ops

pytestmark = pytest.mark.gpu

SCAN_WAIT_CODES = {11, 13, 14, 15, 16, 18, 19}  # producer, MMA and epilogue waits (ssa_select_tc.cu)


def _build(g, dev):
    c, dv = g["case"], g["derived"]
    q = torch.from_numpy(np.ascontiguousarray(g["q"])).to(dev).to(torch.bfloat16)
    k = torch.from_numpy(np.ascontiguousarray(g["k"])).to(dev).to(torch.bfloat16)
    rp = torch.from_numpy(g["rand_proj"]).to(dev).float()
    glob = torch.tensor(g["glob"], dtype=torch.int32, device=dev)
    out = ops.build_graph(q, k, rp, glob, R=c.R, max_p=c.maxP, p_eff=dv["p_eff"], C=dv["C"], T=c.T,
                          A=dv["A"], causal=c.causal and not c.is_cross, is_cross=c.is_cross, K=c.K, window=c.w)
    torch.cuda.synchronize(dev)
    return out


def test_scan_wait_that_runs_out_is_reported_and_the_context_recovers(cuda):
    g = load("c2s_bf16_gqa_causal")  # bf16, d = 128: the tensor-core scan runs
    L = _lib.load()
    L.ssa_device_error(1)
    ref_nb, ref_valid = _build(g, cuda)
    assert L.ssa_device_error(0) == 0
    try:
        L.ssa_debug_set_wait_limit(1)
        _build(g, cuda)  # output undefined: only the error report matters
    finally:
        L.ssa_debug_set_wait_limit(0)
    code = L.ssa_device_error(1)
    assert code in SCAN_WAIT_CODES, code
    nb, valid = _build(g, cuda)
    assert L.ssa_device_error(0) == 0
    assert torch.equal(nb, ref_nb) and torch.equal(valid, ref_valid)
