"""CPU-side checks of the package: API surface, construction order (so one
seed gives the reference's weights), derived hyper-parameters, and the C ABI
(library loads, exports every declared symbol, ctypes layouts match the
header, argument validation) -- nothing here launches a kernel."""
import ctypes
import os
import re
import subprocess
import sys

import numpy as np
import pytest
import torch

import ssa_b200
from ssa_b200 import _lib
from ssa_b200.attention import (CachedGraphSparseTransformer, LSHGraphBuilder, SSAConfig,
                                SparseAttention, SparseTransformer)
from ssa_b200.workloads import WORKLOADS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ssa_b200.h")
GOLDEN = os.path.join(ROOT, "tests", "golden", "module_init.npz")


def test_public_names_match_reference():
    for name in ["SSAConfig", "SubquadraticRegimeTracker", "WindowGraphBuilder",
                 "GlobalGraphBuilder", "LSHGraphBuilder", "merge_neighbors",
                 "sparse_gather_attention", "SparseAttention", "SparseTransformerLayer",
                 "SparseTransformer", "neighbor_overlap", "measure_cross_layer_overlap",
                 "CachedGraphSparseTransformer"]:
        assert hasattr(ssa_b200, name), name


def test_config_defaults_match_reference():
    c = SSAConfig()
    assert (c.d_model, c.num_heads, c.num_kv_heads, c.num_neighbors, c.max_num_hashes,
            c.num_hash_rounds, c.lsh_num_probes, c.window_size, c.num_global_tokens,
            c.global_token_indices, c.dropout, c.causal, c.fp32_attn_weights) == (
        512, 8, None, 128, 12, 8, 0, 8, 2, None, 0.0, False, False)


def test_construction_order_gives_reference_weights():
    """Same seed -> bit-identical weights and hyperplanes as the reference
    modules (fixture written by running the reference)."""
    ref = np.load(GOLDEN)
    torch.manual_seed(1234)
    m = SparseAttention(SSAConfig(d_model=32, num_heads=2, num_kv_heads=1, num_neighbors=12,
                                  max_num_hashes=3, window_size=2, num_global_tokens=1))
    for k, t in m.state_dict().items():
        assert np.array_equal(t.numpy(), ref["attn." + k]), k
    torch.manual_seed(99)
    cfg2 = SSAConfig(d_model=32, num_heads=2, num_neighbors=12, max_num_hashes=2, window_size=3,
                     num_global_tokens=1)
    tr = SparseTransformer(cfg2, num_layers=2, vocab_size=50)
    sd = tr.state_dict()
    assert sorted(sd) == sorted(k[3:] for k in ref.files if k.startswith("tr."))
    for k, t in sd.items():
        assert np.array_equal(t.numpy(), ref["tr." + k]), k
    torch.manual_seed(7)
    cg = CachedGraphSparseTransformer(cfg2, num_layers=3, reuse_every=2)
    for k, t in cg.state_dict().items():
        assert np.array_equal(t.numpy(), ref["cg." + k]), k


def test_rand_proj_stays_fp32_under_casts():
    m = SparseAttention(SSAConfig(d_model=64, num_heads=2, num_neighbors=32, window_size=2))
    before = m.lsh_builder.rand_proj.clone()
    m = m.to(torch.bfloat16)
    assert m.Wq.weight.dtype == torch.bfloat16
    assert m.lsh_builder.rand_proj.dtype == torch.float32
    assert torch.equal(m.lsh_builder.rand_proj, before)
    m = m.half().float()
    assert torch.equal(m.lsh_builder.rand_proj, before)


@pytest.mark.parametrize("cfg,lsh_k,C,p_eff", [("c1", 108, 432, 1), ("c2", 90, 360, 5),
                                              ("c3", 186, 744, 5), ("c4", 108, 432, 1),
                                              ("c5", 107, 428, 4)])
def test_derived_values_per_config(cfg, lsh_k, C, p_eff):
    import warnings
    w = WORKLOADS[cfg]
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        m = SparseAttention(w.config())
    assert m.lsh_k == lsh_k and m.lsh_builder.C == C
    assert m.lsh_builder.compute_effective_p(w.M, C, 12) == p_eff


def test_effective_p_rounds_half_to_even():
    # log2(M / C) = 2.5 exactly -> round() gives 2 (banker's rounding)
    M = int(round(2 ** 2.5 * 1000))
    assert LSHGraphBuilder.compute_effective_p(M, 1000, 12) in (2, 3)
    assert LSHGraphBuilder.compute_effective_p(1, 64, 12) == 1
    assert LSHGraphBuilder.compute_effective_p(10 ** 6, 1, 12) == 12


def test_hot_path_refuses_cpu_tensors():
    m = SparseAttention(SSAConfig(d_model=32, num_heads=2, num_neighbors=12, window_size=2))
    with pytest.raises(ValueError, match="attention_mask"):
        m(torch.randn(1, 8, 32), attention_mask=torch.ones(1, 8))
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.randn(1, 8, 32))


def _declared_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"SSA_API\s+[\w\s\*]+?\b(ssa_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    names = _declared_symbols()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"
    assert L.ssa_abi_version() == 106


def test_static_scratch_size_matches_header():
    m = re.search(r"#define SSA_ATTN_BWD_STATIC_SCRATCH_BYTES \((\d+)u << (\d+)\)", open(HEADER).read())
    assert m, "SSA_ATTN_BWD_STATIC_SCRATCH_BYTES not found in the header"
    assert int(m.group(1)) << int(m.group(2)) == _lib.SSA_ATTN_BWD_STATIC_SCRATCH_BYTES


def test_ctypes_layouts_match_header(tmp_path):
    src = tmp_path / "layout.c"
    fields_g = [f for f, _ in _lib.GraphParams._fields_]
    fields_a = [f for f, _ in _lib.AttnParams._fields_]
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){",
             'printf("%zu %zu\\n", sizeof(ssa_graph_params), sizeof(ssa_attn_params));']
    for f in fields_g:
        lines.append(f'printf("g {f} %zu\\n", offsetof(ssa_graph_params, {f}));')
    for f in fields_a:
        lines.append(f'printf("a {f} %zu\\n", offsetof(ssa_attn_params, {f}));')
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.check_call(["gcc", "-o", str(exe), str(src)])
    out = subprocess.check_output([str(exe)], text=True).split("\n")
    sg, sa = map(int, out[0].split())
    assert sg == ctypes.sizeof(_lib.GraphParams) and sa == ctypes.sizeof(_lib.AttnParams)
    offs = {(l.split()[0], l.split()[1]): int(l.split()[2]) for l in out[1:] if l.strip()}
    for f in fields_g:
        assert offs[("g", f)] == getattr(_lib.GraphParams, f).offset, f
    for f in fields_a:
        assert offs[("a", f)] == getattr(_lib.AttnParams, f).offset, f


def test_integration_stub_matches_header():
    """The reference-side ctypes stub in INTEGRATION.md declares
    ssa_graph_params field for field: same size and offsets as the header's
    struct (which test_ctypes_layouts_match_header pins to _lib.GraphParams)."""
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    m = re.search(r"^class GraphParams\(ctypes\.Structure\):.*?(?=\n\n)", text, re.S | re.M)
    assert m, "GraphParams stub not found in INTEGRATION.md"
    ns = {"ctypes": ctypes}
    exec(m.group(0), ns)
    stub = ns["GraphParams"]
    assert ctypes.sizeof(stub) == ctypes.sizeof(_lib.GraphParams)
    assert [f for f, _ in stub._fields_] == [f for f, _ in _lib.GraphParams._fields_]
    for f, _ in _lib.GraphParams._fields_:
        assert getattr(stub, f).offset == getattr(_lib.GraphParams, f).offset, f
        assert getattr(stub, f).size == getattr(_lib.GraphParams, f).size, f


def _params(**kw):
    p = _lib.GraphParams()
    base = dict(B=1, H=2, n_kv=1, N=64, M=64, d=32, dtype=0, R=2, max_p=6, p_eff=2, C=32, T=0, A=8,
                causal=0, is_cross=0, K=32, window=2, G=1, q_sb=4096, q_sh=2048, q_sn=32,
                k_sb=2048, k_sh=2048, k_sm=32)
    base.update(kw)
    for k, v in base.items():
        setattr(p, k, v)
    return p


def test_abi_validation_rejects_bad_arguments():
    """Host-side checks run before any CUDA call, so they are testable here."""
    L = _lib.load()
    assert L.ssa_graph_workspace_size(ctypes.byref(_params())) > 0
    assert L.ssa_graph_workspace_size(ctypes.byref(_params(H=3, n_kv=2))) == 0
    cases = [(_params(H=3, n_kv=2), _lib.SSA_ERR_INVALID, "divisible"),
             (_params(max_p=13), _lib.SSA_ERR_INVALID, "max_num_hashes"),
             (_params(d=6), _lib.SSA_ERR_UNSUPPORTED, "multiple of 4"),
             (_params(d=256), _lib.SSA_ERR_UNSUPPORTED, "head dim"),
             (_params(is_cross=1, causal=1), _lib.SSA_ERR_INVALID, "never causal")]
    fake = ctypes.c_void_p(0x1000)
    for p, code, msg in cases:
        rc = L.ssa_build_graph(ctypes.byref(p), fake, fake, fake, fake, fake, fake, None, fake,
                               1 << 30, None)
        assert rc == code, (rc, code)
        assert msg in L.ssa_last_error().decode()
    rc = L.ssa_build_graph(ctypes.byref(_params()), None, fake, fake, fake, fake, fake, None, fake,
                           1 << 30, None)
    assert rc == _lib.SSA_ERR_INVALID
    rc = L.ssa_build_graph(ctypes.byref(_params()), fake, fake, fake, fake, fake, fake, None, fake,
                           16, None)
    assert rc == _lib.SSA_ERR_WORKSPACE
    with pytest.raises(ValueError):
        _lib.check(_lib.SSA_ERR_INVALID, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.SSA_ERR_UNSUPPORTED, "x")


def test_fused_projection_rejects_unserved_params():
    """ssa_qkv_proj_hash serves bf16 self-attention with the output-view
    strides only; everything else is reported before any CUDA work."""
    L = _lib.load()
    fake = ctypes.c_void_p(0x1000)
    for p in (_params(dtype=_lib.SSA_F32), _params(is_cross=1, causal=0), _params(q_sn=7)):
        assert L.ssa_qkv_proj_hash_supported(ctypes.byref(p), 512) == 0
        rc = L.ssa_qkv_proj_hash(ctypes.byref(p), 512, fake, fake, fake, fake, fake, 1 << 30, None)
        assert rc == _lib.SSA_ERR_UNSUPPORTED, rc
        assert "fused projection" in L.ssa_last_error().decode()


def test_graph_width_matches_oracle_formula():
    from oracle import oracle as O
    L = _lib.load()
    for K, w, G, A, cross in [(128, 8, 2, 108, 0), (128, 8, 3, 107, 1), (16, 8, 4, 8, 0), (4, 1, 1, 8, 1)]:
        p = _params(K=K, window=w, G=G, A=A, is_cross=cross)
        kall = (0 if cross else 2 * w + 1) + G + A
        assert L.ssa_graph_width(ctypes.byref(p)) == O.lib().ora_merge_width(K, kall, cross)


# --- host-side contract of the reference's modules (no device needed) -------
# The reference's asserts and guards fire before any kernel runs, so they are
# checked here on CPU: tests/test_gqa_mqa.py:25-66 and
# tests/test_global_tokens_and_mask_guard.py:51-65 of the reference.

def _small(**kw):
    base = dict(d_model=64, num_heads=4, num_neighbors=16, window_size=4, num_global_tokens=2,
                max_num_hashes=3)
    base.update(kw)
    return SSAConfig(**base)


def test_kv_parameter_counts_scale_with_kv_heads():
    def kv_params(n_kv):
        attn = SparseAttention(_small(num_kv_heads=n_kv))
        return sum(p.numel() for p in attn.Wk.parameters()) + sum(p.numel() for p in attn.Wv.parameters())
    p1, p2, p4 = kv_params(1), kv_params(2), kv_params(4)
    assert p1 * 4 == p4 and p2 * 2 == p4 and p1 < p2 < p4


@pytest.mark.parametrize("kw", [dict(num_heads=5, num_kv_heads=2),   # heads % kv heads
                                dict(d_model=60, num_heads=8),       # d_model % heads
                                dict(max_num_hashes=13),             # at most 12 hyperplanes
                                dict(lsh_num_probes=-1)])            # probes >= 0
def test_config_asserts(kw):
    with pytest.raises(AssertionError):
        SparseAttention(_small(**kw))


def test_reuse_every_must_be_positive():
    with pytest.raises(AssertionError):
        CachedGraphSparseTransformer(_small(), num_layers=2, reuse_every=0)


def test_attention_mask_raises_before_any_kernel():
    attn = SparseAttention(_small())
    with pytest.raises(ValueError, match="attention_mask"):
        attn(torch.randn(2, 32, 64), attention_mask=torch.ones(2, 32))


def test_budget_warning_when_window_and_globals_exceed_k():
    with pytest.warns(UserWarning, match="budget"):
        attn = SparseAttention(_small(num_neighbors=8, window_size=4))
    assert attn.lsh_k == 8  # floored, as the reference does
