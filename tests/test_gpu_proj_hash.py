"""Fused QKV projection + hash (ssa_qkv_proj_hash) against torch and against
the unfused graph build.

  * qkv = x [Wq; Wk; Wv]^T in bf16 matches an fp32 matmul of the same bf16
    operands within bf16 rounding (2e-2 of the largest value, the contract's
    bf16 band), and torch's own bf16 Linear likewise;
  * the graph built from the fused kernel's hash state
    (ssa_build_graph_prehashed) equals ssa_build_graph on the q / k views of
    its output, bit for bit;
  * SparseAttention with fuse_qkv set takes the fused path for bf16
    self-attention, and its output and gradients match the unfused module's
    within the bf16 band;
  * shapes the kernel does not serve are reported as such (None).
"""
import zlib

import pytest
import torch

from oracle import oracle as O
from parity import record

from ssa_b200 import _lib, ops
from ssa_b200.attention import SparseAttention, SSAConfig

pytestmark = pytest.mark.gpu

# name, B, N, d_model, H, n_kv, K, window, G, R, maxP, T
CFGS = [
    ("gqa_d128", 2, 1024, 1024, 8, 2, 128, 16, 4, 8, 12, 0),
    ("mha_d64_probes2", 1, 2048, 512, 8, 8, 96, 8, 2, 8, 12, 2),
    ("mqa_d64_probe1_partial_tile", 2, 512, 768, 12, 1, 64, 4, 2, 8, 12, 1),  # 896 output columns
]


def _setup(cfg, dev):
    name, B, N, dm, H, n_kv, K, w, G, R, maxP, T = cfg
    d = dm // H
    g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
    x = torch.randn(B, N, dm, generator=g).to(dev, torch.bfloat16)
    bound = dm ** -0.5
    W = ((torch.rand((H + 2 * n_kv) * d, dm, generator=g) * 2 - 1) * bound).to(dev, torch.bfloat16)
    rp = torch.randn(R, maxP, d, generator=g).to(dev)
    dv = O.derived(K, w, G, R, maxP, T, N)
    glob = torch.arange(G, dtype=torch.int32, device=dev)
    kw = dict(H=H, n_kv=n_kv, R=R, max_p=maxP, p_eff=dv["p_eff"], C=dv["C"], T=T, A=dv["A"], causal=True,
              K=K, window=w)
    return x, W, rp, glob, kw


@pytest.mark.parametrize("cfg", CFGS, ids=[c[0] for c in CFGS])
def test_fused_projection_and_graph(cfg, cuda):
    x, W, rp, glob, kw = _setup(cfg, cuda)
    L = _lib.load()
    L.ssa_debug_hash_recomputed(1)
    res = ops.qkv_project_hash(x, W, rp, glob, **kw)
    assert res is not None, "the fused path should serve this shape"
    qkv, state = res
    torch.cuda.synchronize()
    assert L.ssa_device_error(1) == 0
    ref = x.float() @ W.float().t()
    scale = ref.abs().max().item()
    err = (qkv.float() - ref).abs().max().item() / scale
    err_torch = (qkv.float() - torch.nn.functional.linear(x, W).float()).abs().max().item() / scale
    exact_frac = (qkv == ref.to(torch.bfloat16)).float().mean().item()
    print(f"{cfg[0]}: max err vs fp32 {err:.2e}, vs torch bf16 {err_torch:.2e}, "
          f"bit-equal to round(fp32) {100 * exact_frac:.2f} %")
    assert err <= 2e-2 and err_torch <= 2e-2
    q, k, v = ops.split_qkv(qkv, kw["H"], kw["n_kv"])
    nb_f, va_f = ops.build_graph_prehashed(q, k, state)
    nb_u, va_u = ops.build_graph(q, k, rp, glob, R=kw["R"], max_p=kw["max_p"], p_eff=kw["p_eff"], C=kw["C"],
                                 T=kw["T"], A=kw["A"], causal=True, is_cross=False, K=kw["K"],
                                 window=kw["window"])
    torch.cuda.synchronize()
    assert L.ssa_device_error(1) == 0
    assert torch.equal(va_f, va_u)
    assert torch.equal(nb_f[va_u.bool()], nb_u[va_u.bool()])
    record("proj_hash_" + cfg[0], proj_rel_err=err, graph_rows=va_u.shape[0] * va_u.shape[1] * va_u.shape[2],
           graph_rows_mismatched=0)


def test_unserved_shapes_return_none(cuda):
    cfg = ("odd_n", 1, 1000, 512, 8, 2, 64, 4, 2, 8, 12, 0)  # N % 128 != 0
    x, W, rp, glob, kw = _setup(cfg, cuda)
    assert ops.qkv_project_hash(x, W, rp, glob, **kw) is None


def test_module_uses_fused_path_and_matches_unfused(cuda):
    cfg = SSAConfig(d_model=512, num_heads=8, num_kv_heads=2, num_neighbors=96, window_size=8,
                    num_global_tokens=2, num_hash_rounds=8, max_num_hashes=12, lsh_num_probes=1, causal=True)
    torch.manual_seed(0)
    m = SparseAttention(cfg).to(cuda).to(torch.bfloat16)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 1024, 512, generator=g).to(cuda, torch.bfloat16)
    outs, grads = [], []
    for fuse in (True, False):
        m.fuse_qkv = fuse
        xi = x.clone().requires_grad_(True)
        calls0 = _lib.load().ssa_kernel_launches()
        out, _ = m(xi)
        out.float().pow(2).sum().backward()
        outs.append(out.detach().float())
        grads.append([xi.grad.float()] + [p.grad.float().clone() for p in (m.Wq.weight, m.Wk.weight, m.Wv.weight)])
        for p in m.parameters():
            p.grad = None
        assert _lib.load().ssa_kernel_launches() > calls0
    rel = lambda a, b: ((a - b).norm() / b.norm()).item()
    assert rel(outs[0], outs[1]) <= 2e-2, rel(outs[0], outs[1])
    for a, b in zip(grads[0], grads[1]):
        assert rel(a, b) <= 2e-2, rel(a, b)
