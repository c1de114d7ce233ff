"""Host logic of the multi-GPU partitioning (ssa_b200.sharding), on CPU.

The partition helpers are checked directly. The sharded runners then run
as gloo ranks (world_size 2, 3 and 4), with the oracle injected as the per-slice
compute. Their assembled outputs must equal the oracle run on the whole
problem. The oracle is the checker here: the runners' own compute is the
CUDA ops, which the GPU tests cover.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from ssa_b200.sharding import GroupSharded, RowSharded, group_slices, split_range

CFG = dict(K=24, w=2, G=2, glob_idx=None, R=3, maxP=6, T=1)


@pytest.mark.parametrize("total,world", [(32, 8), (32, 3), (7, 4), (5, 8), (1, 1)])
def test_split_range_covers_once(total, world):
    seen = []
    for r in range(world):
        lo, hi = split_range(total, world, r)
        assert 0 <= lo <= hi <= total
        seen.extend(range(lo, hi))
    assert seen == list(range(total))
    sizes = [split_range(total, world, r)[1] - split_range(total, world, r)[0] for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("B,n_kv,world", [(4, 8, 8), (4, 8, 3), (1, 16, 8), (8, 1, 8), (2, 3, 4)])
def test_group_slices_partition_units(B, n_kv, world):
    units = []
    for r in range(world):
        for s in group_slices(B, n_kv, world, r):
            assert 0 <= s.g0 < s.g1 <= n_kv and 0 <= s.b0 < s.b1 <= B
            assert s.b1 - s.b0 == 1 or (s.g0, s.g1) == (0, n_kv)
            units.extend((b, g) for b in range(s.b0, s.b1) for g in range(s.g0, s.g1))
    assert units == [(b, g) for b in range(B) for g in range(n_kv)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(B=2, H=4, n_kv=2, N=64, d=16):
    g = torch.Generator().manual_seed(3)
    q = torch.randn(B, H, N, d, generator=g)
    k = torch.randn(B, n_kv, N, d, generator=g)
    v = torch.randn(B, n_kv, N, d, generator=g)
    planes = torch.nn.functional.normalize(torch.randn(CFG["R"], CFG["maxP"], d, generator=g), dim=-1)
    return q, k, v, planes


def _oracle_fns(planes, n_kv_total_unused=None):
    from oracle import oracle as ora

    def graph(q, k, M, causal, is_cross, q_row0):
        # Rows of a graph build are independent given all keys: place the
        # slice at its sequence positions in a zero query tensor of full
        # length, build, and keep the slice's rows.
        q = q.contiguous().numpy()
        B, H, n, d = q.shape
        full = np.zeros((B, H, q_row0 + n, d), dtype=np.float32)
        full[:, :, q_row0:q_row0 + n] = q
        nb, valid = ora.build_graph(full, k.contiguous().numpy(), planes.numpy(), n_kv=k.shape[1],
                                    causal=causal, is_cross=is_cross, **CFG)
        return torch.from_numpy(np.ascontiguousarray(nb[:, :, q_row0:])), \
            torch.from_numpy(np.ascontiguousarray(valid[:, :, q_row0:]))

    def attn(q, k, v, nb, valid):
        out, _ = ora.attn_fwd(q.contiguous().numpy(), k.contiguous().numpy(), v.contiguous().numpy(),
                              nb.numpy(), valid.numpy(), scale=q.shape[-1] ** -0.5, lowp=False, fp32_w=False)
        return torch.from_numpy(out)

    return graph, attn


def _worker(rank, world, port, mode, causal, result_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, planes = _problem()
        graph, attn = _oracle_fns(planes)
        B, H, N, d = q.shape
        n_kv = k.shape[1]
        if mode == "rows":
            runner = RowSharded(None, N, world, rank, causal=causal, graph_fn=graph, attn_fn=attn)
            r0, r1 = runner.rows
            k_seq = k.permute(2, 0, 1, 3)[r0:r1].contiguous()  # this rank's key rows, sequence-major
            v_seq = v.permute(2, 0, 1, 3)[r0:r1].contiguous()
            kg, vg = runner.gather_kv(k_seq, v_seq)
            assert torch.equal(kg, k) and torch.equal(vg, v), "all-gathered K/V differ from the full tensors"
            out_local = runner.step(q[:, :, r0:r1], k_seq, v_seq)
            parts = [torch.empty_like(out_local) for _ in range(world)]
            dist.all_gather(parts, out_local.contiguous())
            out = torch.cat(parts, dim=2)
        else:
            runner = GroupSharded(None, world, rank, causal=causal, graph_fn=graph, attn_fn=attn)
            out = torch.zeros(B, H, N, d)
            rep = H // n_kv
            for s, o in runner.step(q, k, v):
                out[s.b0:s.b1, s.g0 * rep:s.g1 * rep] = o
            dist.all_reduce(out)  # every element is written by exactly one rank
        if rank == 0:
            torch.save(out, result_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode,causal,world", [("rows", True, 2), ("rows", False, 2), ("groups", True, 2),
                                               ("rows", True, 4), ("groups", False, 3)])
def test_sharded_runners_match_unsharded(tmp_path, mode, causal, world):
    result = str(tmp_path / "out.pt")
    mp.spawn(_worker, args=(world, _free_port(), mode, causal, result), nprocs=world, join=True)
    q, k, v, planes = _problem()
    graph, attn = _oracle_fns(planes)
    nb, valid = graph(q, k, q.shape[2], causal, False, 0)
    ref = attn(q, k, v, nb, valid)
    out = torch.load(result)
    assert torch.equal(out, ref)


def _leaving_worker(rank, world, port, result_path):
    """Rank 1 leaves before the step's K/V all-gather (between steps, with
    nothing in flight); rank 0 must get an error from the collective within
    the process group's timeout rather than wait for ever."""
    import datetime
    import time

    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    q, k, v, planes = _problem()
    N = q.shape[2]
    runner = RowSharded(None, N, world, rank, causal=True, graph_fn=None, attn_fn=None)
    r0, r1 = runner.rows
    k_seq = k.permute(2, 0, 1, 3)[r0:r1].contiguous()
    v_seq = v.permute(2, 0, 1, 3)[r0:r1].contiguous()
    if rank == 1:
        dist.destroy_process_group()
        return
    t0 = time.monotonic()
    outcome = "completed"
    try:
        runner.gather_kv(k_seq, v_seq)
    except Exception as e:  # gloo reports the missing peer as a RuntimeError
        outcome = f"raised {type(e).__name__}"
    with open(result_path, "w") as f:
        f.write(f"{outcome} {time.monotonic() - t0:.1f}")


def test_rank_leaving_surfaces_as_error_not_hang(tmp_path):
    result = str(tmp_path / "outcome.txt")
    mp.spawn(_leaving_worker, args=(2, _free_port(), result), nprocs=2, join=True)
    outcome, seconds = open(result).read().rsplit(" ", 1)
    print("surviving rank:", outcome, seconds, "s")
    assert outcome.startswith("raised"), outcome
    assert float(seconds) < 60.0
