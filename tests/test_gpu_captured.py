"""CapturedStep (ssa_b200/captured.py): the graph build + gather attention
captured as one CUDA graph gives exactly the eager step's output, at capture
and on replays with new inputs copied in, and it replays the package's own
kernels (the launch counter moves only while capturing)."""
import pytest
import torch

from ssa_b200 import _lib, ops
from ssa_b200.attention import SparseAttention, SSAConfig
from ssa_b200.captured import CapturedStep

pytestmark = pytest.mark.gpu

# name, dtype, B, N, d_model, H, n_kv, K, window, G, causal
CFGS = [
    ("c1_like_fp32", torch.float32, 2, 1024, 512, 8, 8, 128, 8, 2, True),
    ("gqa_bf16_d128", torch.bfloat16, 1, 2048, 1024, 8, 2, 128, 16, 4, True),
]


def _eager(m, q, k, v, causal):
    nb, valid = m._graph(q, k, k.shape[2], causal, False)
    out, _ = ops.attn_fwd(q, k, v, nb, valid, m.scale, m.config.fp32_attn_weights, want_lse=False)
    return out


def _qkv(m, cfg, seed, dev):
    name, dt, B, N, dm, H, n_kv, *_ = cfg
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, N, dm, generator=g).to(dev, dt)
    with torch.no_grad():
        return m._split_q(m.Wq(x)), m._split_kv_grouped(m.Wk(x)), m._split_kv_grouped(m.Wv(x))


@pytest.mark.parametrize("cfg", CFGS, ids=[c[0] for c in CFGS])
def test_captured_step_equals_eager(cfg, cuda):
    name, dt, B, N, dm, H, n_kv, K, w, G, causal = cfg
    conf = SSAConfig(d_model=dm, num_heads=H, num_kv_heads=n_kv, num_neighbors=K, window_size=w,
                     num_global_tokens=G, num_hash_rounds=8, max_num_hashes=12, lsh_num_probes=0, causal=causal)
    torch.manual_seed(0)
    m = SparseAttention(conf).to(cuda).to(dt).eval()
    q, k, v = _qkv(m, cfg, 1, cuda)
    L = _lib.load()
    with torch.no_grad():
        ref = _eager(m, q, k, v, causal)
        cs = CapturedStep(m, q, k, v)
        n0 = L.ssa_kernel_launches()
        out = cs().clone()
        torch.cuda.synchronize()
        assert L.ssa_kernel_launches() == n0, "a replay must not go through the eager launch path"
        assert torch.equal(out, ref)
        q2, k2, v2 = _qkv(m, cfg, 2, cuda)
        ref2 = _eager(m, q2, k2, v2, causal)
        out2 = cs(q2, k2, v2).clone()
        torch.cuda.synchronize()
        assert L.ssa_device_error(1) == 0
        assert torch.equal(out2, ref2)
        assert not torch.equal(out2, out)
        with pytest.raises(ValueError):
            cs(q2[:, :, : N // 2])
