"""Tensor-core hash (ssa_hash_tc.cu) against the fp32 FMA hash kernels.

bf16 inputs with head dim 64 or 128 are hashed on the tensor cores, with an
exact fp32 recompute of every projection the certification bound cannot
decide. The ids -- and so the whole graph -- must equal the FMA kernels'
bit for bit:
  * graphs built with the tensor-core hash (default constant c, and c = 1,
    which sends every projection to the recompute) equal the FMA-hash graph;
  * the tensor-core projections lie within c |x|_2 max_j |P_j|_2 / 8 of the
    exact (fp64) projections, i.e. the bound has a margin of at least 8;
  * the recompute stays rare at the default c.
"""
import ctypes
import zlib

import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import record

from ssa_b200 import _lib, ops

pytestmark = pytest.mark.gpu

C_DEFAULT = 2.0 ** -14

# name, B, H, n_kv, N, d, K, window, G, R, maxP, T, causal, clustered
CFGS = [
    ("gqa_d128_causal", 2, 8, 2, 4096, 128, 128, 16, 4, 8, 12, 0, True, False),
    ("mha_d128_probes2_clusters", 1, 4, 4, 8192, 128, 256, 32, 4, 8, 12, 2, False, True),
    ("mqa_d64_probe1", 2, 8, 1, 4096, 64, 128, 8, 3, 8, 12, 1, False, False),
    ("d64_r16_probes3", 1, 4, 2, 2048, 64, 96, 8, 2, 16, 10, 3, True, True),
]


def _inputs(cfg, dev):
    name, B, H, n_kv, N, d, K, w, G, R, maxP, T, causal, clustered = cfg
    g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
    if clustered:  # mixture of isotropic Gaussian clusters: skewed buckets, near-ties
        centers = torch.randn(64, d, generator=g)
        def draw(*shape):
            idx = torch.randint(0, 64, shape[:-1], generator=g)
            return centers[idx] + 0.3 * torch.randn(*shape, generator=g)
        q, k = draw(B, H, N, d), draw(B, n_kv, N, d)
    else:
        q, k = torch.randn(B, H, N, d, generator=g), torch.randn(B, n_kv, N, d, generator=g)
    rp = torch.randn(R, maxP, d, generator=g)
    dv = O.derived(K, w, G, R, maxP, T, N)
    glob = torch.arange(G, dtype=torch.int32)
    return (q.to(dev, torch.bfloat16), k.to(dev, torch.bfloat16), rp.to(dev), glob.to(dev), dv)


def _build(cfg, q, k, rp, glob, dv):
    name, B, H, n_kv, N, d, K, w, G, R, maxP, T, causal, clustered = cfg
    return ops.build_graph(q, k, rp, glob, R=R, max_p=maxP, p_eff=dv["p_eff"], C=dv["C"], T=T,
                           A=dv["A"], causal=causal, is_cross=False, K=K, window=w)


def _set_hash(use_tc, c):
    L = _lib.load()
    assert L.ssa_debug_set_hash(use_tc, c) == 0


@pytest.fixture
def hash_mode():
    yield _set_hash
    _set_hash(1, 0.0)
    _lib.load().ssa_debug_hash_dump(None, 0)


@pytest.mark.parametrize("cfg", CFGS, ids=[c[0] for c in CFGS])
def test_tensor_core_hash_graph_equals_fma_hash(cfg, cuda, hash_mode):
    q, k, rp, glob, dv = _inputs(cfg, cuda)
    L = _lib.load()
    hash_mode(0, 0.0)
    nb_f, va_f = _build(cfg, q, k, rp, glob, dv)
    hash_mode(1, 0.0)
    L.ssa_debug_hash_recomputed(1)
    nb_t, va_t = _build(cfg, q, k, rp, glob, dv)
    torch.cuda.synchronize()
    rec = L.ssa_debug_hash_recomputed(1)
    hash_mode(1, 1.0)  # every projection recomputed in fp32
    nb_a, va_a = _build(cfg, q, k, rp, glob, dv)
    torch.cuda.synchronize()
    rec_all = L.ssa_debug_hash_recomputed(1)
    assert L.ssa_device_error(1) == 0
    assert torch.equal(va_t, va_f) and torch.equal(nb_t[va_f.bool()], nb_f[va_f.bool()])
    assert torch.equal(va_a, va_f) and torch.equal(nb_a[va_f.bool()], nb_f[va_f.bool()])
    name, B, H, n_kv, N, d, K, w, G, R, maxP, T, causal, clustered = cfg
    items = (B * H * N + B * n_kv * N) * R  # (row, round) items: queries and keys
    assert rec_all == items, (rec_all, items)
    frac = rec / items
    record("hash_tc_" + name, hash_items=items, hash_items_recomputed=rec)
    print(f"{name}: recomputed {rec} of {items} (row, round) items ({100 * frac:.3f} %)")
    assert frac < 0.05


@pytest.mark.parametrize("cfg", CFGS, ids=[c[0] for c in CFGS])
def test_tensor_core_projection_error_within_bound(cfg, cuda, hash_mode):
    name, B, H, n_kv, N, d, K, w, G, R, maxP, T, causal, clustered = cfg
    q, k, rp, glob, dv = _inputs(cfg, cuda)
    p = dv["p_eff"]
    L = _lib.load()
    dump = torch.full((B * H * N * R * p,), float("nan"), dtype=torch.float32, device=cuda)
    assert L.ssa_debug_hash_dump(ctypes.c_void_p(dump.data_ptr()), dump.numel()) == 0
    _build(cfg, q, k, rp, glob, dv)
    torch.cuda.synchronize()
    assert L.ssa_debug_hash_dump(None, 0) == 0
    x = q.reshape(-1, d).double()
    planes = rp[:, :p, :].double()                                    # (R, p, d)
    exact = torch.einsum("nd,rpd->nrp", x, planes)                    # (rows, R, p)
    got = dump.view(-1, R, p).double()
    assert not torch.isnan(got).any()
    bound = x.norm(dim=1)[:, None] * planes.norm(dim=2).max(dim=1).values[None, :]  # (rows, R)
    ratio = ((got - exact).abs().amax(dim=2) / bound.clamp_min(1e-30)).max().item()
    record("hash_tc_" + name, hash_error_ratio_max=ratio)
    print(f"{name}: max |v_tc - v_exact| / (|x| max|P|) = {ratio:.3e} (c = {C_DEFAULT:.3e})")
    assert ratio <= C_DEFAULT / 8


def test_fma_hash_still_serves_fp32(cuda, hash_mode):
    # fp32 inputs never take the tensor-core hash; the recompute counter stays 0
    L = _lib.load()
    cfg = CFGS[2]
    q, k, rp, glob, dv = _inputs(cfg, cuda)
    L.ssa_debug_hash_recomputed(1)
    _build(cfg, q.float(), k.float(), rp, glob, dv)
    torch.cuda.synchronize()
    assert L.ssa_debug_hash_recomputed(1) == 0
