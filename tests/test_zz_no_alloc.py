"""ssa_attn_bwd_noalloc: the attention backward whose scratch is a static
device array instead of a caller workspace. Called through the C ABI and
compared with ssa_attn_bwd (caller workspace) on the same inputs, on two
calls in a row; oversized problems are rejected before any launch.

The file name sorts last so that the first call of the process may come
either first (run alone) or after every other test.
"""
import ctypes

import pytest
import torch

from ssa_b200 import _lib, ops

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def _problem(dev, dtype, B=2, H=4, n_kv=2, N=192, M=256, d=64, Kn=40):
    g = torch.Generator(device="cpu").manual_seed(7)
    q = torch.randn(B, H, N, d, generator=g).to(device=dev, dtype=dtype)
    k = torch.randn(B, n_kv, M, d, generator=g).to(device=dev, dtype=dtype)
    v = torch.randn(B, n_kv, M, d, generator=g).to(device=dev, dtype=dtype)
    nb = torch.randint(0, M, (B, H, N, Kn), generator=g, dtype=torch.int32).to(dev)
    valid = (torch.rand(B, H, N, Kn, generator=g) < 0.8)
    valid[..., 0] = True
    valid = valid.to(dev)
    dO = torch.randn(B, H, N, d, generator=g).to(device=dev, dtype=dtype)
    return q, k, v, nb, valid, dO


def _params(q, k, v, nb, dO, scale):
    p = ops._attn_params(q, k, v, nb, scale, False, tuple(dO.stride()[:3]))
    p.q_sb, p.q_sh, p.q_sn = q.stride()[:3]
    p.k_sb, p.k_sh, p.k_sm = k.stride()[:3]
    p.v_sb, p.v_sh, p.v_sm = v.stride()[:3]
    return p


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_workspace_backward(cuda, dtype):
    q, k, v, nb, valid, dO = _problem(cuda, dtype)
    scale = q.shape[-1] ** -0.5
    _, lse = ops.attn_fwd(q, k, v, nb, valid, scale, False, want_lse=True)
    dq_ref, dk_ref, dv_ref = ops.attn_bwd(q, k, v, nb, valid, dO, lse, scale, False)

    L = _lib.load()
    p = _params(q, k, v, nb, dO, scale)
    valid_u8 = valid.contiguous().view(torch.uint8)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    assert L.ssa_attn_bwd_workspace_size(ctypes.byref(p)) <= _lib.SSA_ATTN_BWD_STATIC_SCRATCH_BYTES
    for call in range(2):
        dq = torch.full_like(dO, float("nan"))
        dk = torch.full_like(k, float("nan"))
        dv = torch.full_like(v, float("nan"))
        rc = L.ssa_attn_bwd_noalloc(ctypes.byref(p), ops._ptr(q), ops._ptr(k), ops._ptr(v), ops._ptr(nb),
                                    ops._ptr(valid_u8), ops._ptr(dO), ops._ptr(lse), ops._ptr(dq),
                                    ops._ptr(dk), ops._ptr(dv), stream)
        assert rc == _lib.SSA_OK, L.ssa_last_error().decode()
        torch.cuda.synchronize(cuda)
        for got, ref, name in ((dq, dq_ref, "dq"), (dk, dk_ref, "dk"), (dv, dv_ref, "dv")):
            assert torch.isfinite(got.float()).all(), f"call {call}: {name} not fully written"
            assert _rel(got, ref) <= TOL[dtype], f"call {call}: {name} rel err {_rel(got, ref):.3e}"
    assert L.ssa_device_error(1) == 0


def test_noalloc_rejects_oversized_problem(cuda):
    q, k, v, nb, valid, dO = _problem(cuda, torch.float32)
    scale = q.shape[-1] ** -0.5
    lse = torch.zeros(q.shape[:3], dtype=torch.float32, device=cuda)
    p = _params(q, k, v, nb, dO, scale)
    p.N = 1 << 20  # 2*4*2^20*40 edges: far beyond the static scratch
    L = _lib.load()
    assert L.ssa_attn_bwd_workspace_size(ctypes.byref(p)) > _lib.SSA_ATTN_BWD_STATIC_SCRATCH_BYTES
    valid_u8 = valid.contiguous().view(torch.uint8)
    rc = L.ssa_attn_bwd_noalloc(ctypes.byref(p), ops._ptr(q), ops._ptr(k), ops._ptr(v), ops._ptr(nb),
                                ops._ptr(valid_u8), ops._ptr(dO), ops._ptr(lse), ops._ptr(dO),
                                ops._ptr(k), ops._ptr(v), ctypes.c_void_p(0))
    assert rc == _lib.SSA_ERR_WORKSPACE
    msg = L.ssa_last_error().decode()
    assert "static scratch" in msg and str(_lib.SSA_ATTN_BWD_STATIC_SCRATCH_BYTES) in msg


@pytest.mark.parametrize("d", [64, 128])
def test_noalloc_limit_is_the_workspace_size(cuda, d):
    """The largest problem whose scratch fits runs and matches the workspace
    path; one query row more is rejected (the limit the header states is
    ssa_attn_bwd_workspace_size <= SSA_ATTN_BWD_STATIC_SCRATCH_BYTES)."""
    L = _lib.load()
    B, H, n_kv, M, Kn = 1, 8, 2, 8192, 128
    probe = torch.empty(1, H, 1, d, device=cuda, dtype=torch.bfloat16)
    kv = torch.empty(B, n_kv, M, d, device=cuda, dtype=torch.bfloat16)

    def need(N):
        p = _params(probe.expand(B, H, N, d), kv, kv,
                    torch.empty(B, H, N, Kn, device=cuda, dtype=torch.int32),
                    torch.empty(B, H, N, d, device=cuda, dtype=torch.bfloat16), 1.0)
        return L.ssa_attn_bwd_workspace_size(ctypes.byref(p))
    lo, hi = 1, 1 << 16
    while lo < hi:
        mid = (lo + hi + 1) // 2
        lo, hi = (mid, hi) if need(mid) <= _lib.SSA_ATTN_BWD_STATIC_SCRATCH_BYTES else (lo, mid - 1)
    N = lo
    assert 2.0e6 <= B * H * N * Kn <= 2.6e6  # the header's "about 2.5 / 2.3 million edges"
    q, k, v, nb, valid, dO = _problem(cuda, torch.bfloat16, B=B, H=H, n_kv=n_kv, N=N, M=M, d=d, Kn=Kn)
    scale = d ** -0.5
    _, lse = ops.attn_fwd(q, k, v, nb, valid, scale, False, want_lse=True)
    ref = ops.attn_bwd(q, k, v, nb, valid, dO, lse, scale, False)
    p = _params(q, k, v, nb, dO, scale)
    valid_u8 = valid.contiguous().view(torch.uint8)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    outs = [torch.full_like(dO, float("nan")), torch.full_like(k, float("nan")), torch.full_like(v, float("nan"))]
    rc = L.ssa_attn_bwd_noalloc(ctypes.byref(p), ops._ptr(q), ops._ptr(k), ops._ptr(v), ops._ptr(nb),
                                ops._ptr(valid_u8), ops._ptr(dO), ops._ptr(lse), *[ops._ptr(t) for t in outs],
                                stream)
    assert rc == _lib.SSA_OK, L.ssa_last_error().decode()
    torch.cuda.synchronize(cuda)
    for got, r in zip(outs, ref):
        assert _rel(got, r) <= TOL[torch.bfloat16]
    p.N = N + 1
    assert need(N + 1) > _lib.SSA_ATTN_BWD_STATIC_SCRATCH_BYTES
    rc = L.ssa_attn_bwd_noalloc(ctypes.byref(p), ops._ptr(q), ops._ptr(k), ops._ptr(v), ops._ptr(nb),
                                ops._ptr(valid_u8), ops._ptr(dO), ops._ptr(lse), *[ops._ptr(t) for t in outs],
                                stream)
    assert rc == _lib.SSA_ERR_WORKSPACE
    assert L.ssa_device_error(1) == 0
