#!/usr/bin/env python
"""Benchmark of the sparse-attention hot path: graph build + gather attention
forward (the reference's "fwd+graph" metric) on one of the BASELINE
workloads, default the headline GQA config c2 (B=4, N=8192, 32 q / 8 kv
heads, d=128, K=128, bf16).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2]
    python bench.py --impl reference ...     # CPU reference arm (oracle port)

One step = SparseAttention's graph build (hash, buckets, candidate scan +
top-k, merge) and gather attention over q/k/v already resident in HBM.
Under torchrun the ranks split ONE job (strong scaling): (batch, kv-head)
groups with no collective, or query rows with one NCCL all-gather of K/V for
the long-context config; the step time is the maximum over ranks. L2 is
flushed (a 256 MB write) between timed steps; every step is timed with CUDA
events on the launching stream.

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import csv
import datetime
import io
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sparse-attn fwd+graph tokens/s/GPU at N=8192,K=128; % HBM roofline"
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "traffic.json")


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--mode", default="fwd", choices=["fwd", "train", "model", "proj"],
                    help="fwd: graph build + attention forward (the headline metric); train: "
                         "graph build + attention forward + backward (one layer's attention core); "
                         "model: the training-config model step (c4: 6-layer SparseTransformer with "
                         "its vocab embedding, forward + out.sum().backward(), and the same with "
                         "CachedGraphSparseTransformer(reuse_every=4) behind an embedding); "
                         "proj: the fused QKV projection + hash (ssa_qkv_proj_hash) and the graph "
                         "built from it, against torch Linear + the graph build, from x")
    ap.add_argument("--impl", default="ssa", choices=["ssa", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-chunks", type=int, default=8,
                    help="e2e: split the rank's (batch, kv-head) slices into about this many pipeline "
                         "chunks (halving kv-head ranges down to two heads), with tapered first and last chunks")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's batch size (profiling a smaller case)")
    ap.add_argument("--shard", default="auto", choices=["auto", "groups", "rows"],
                    help="multi-GPU partitioning (auto: query rows for c3, (batch, kv-head) groups otherwise)")
    ap.add_argument("--baseline-slices", type=int, default=2,
                    help="(batch, kv-group) slices in the CPU baseline sample")
    ap.add_argument("--no-long-context", action="store_true",
                    help="skip the second measurement of the long-context config c3 on the same GPUs")
    ap.add_argument("--no-other-workloads", action="store_true",
                    help="skip the c1 / c5 / c4 objects of the default run")
    ap.add_argument("--no-graph-profile", action="store_true",
                    help="skip the per-stage timing of the graph build after the timed steps")
    return ap.parse_args(argv)


def hbm_peak():
    try:
        with open(PEAKS_FILE) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def peaks():
    """hbm_gbs and bf16_tflops_sustained: MEASURED_PEAKS.json, else the pool's
    fallback figures."""
    try:
        with open(PEAKS_FILE) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops_sustained": float(d["bf16_tflops_sustained"]),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="ssa_clocks_", suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        rows = []
        with open(self.path) as f:
            for r in csv.reader(f):
                if len(r) >= 9:
                    rows.append([x.strip() for x in r])
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def dist_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port on a bounded sample of the same workload
# ---------------------------------------------------------------------------
def cpu_sample(w, m, q, k, v, slices: int):
    """Runs the oracle's build_graph + attention forward on `slices`
    (batch, kv-group) slices; returns (seconds, description, threads)."""
    from oracle import oracle as O
    rep = w.H // w.n_kv
    lsh = m.lsh_builder
    rp = lsh.rand_proj.detach().cpu().float().numpy()
    glob_idx = list(w.glob) if w.glob else None
    work = []
    for s in range(slices):
        b, g = divmod(s, w.n_kv)
        b = b % w.B
        work.append((q[b:b + 1, g * rep:(g + 1) * rep].float().contiguous().cpu().numpy(),
                     k[b:b + 1, g:g + 1].float().contiguous().cpu().numpy(),
                     v[b:b + 1, g:g + 1].float().contiguous().cpu().numpy()))
    t0 = time.perf_counter()
    for qs, ks, vs in work:
        nb, va = O.build_graph(qs, ks, rp, n_kv=1, K=w.K, w=w.window, G=w.G, glob_idx=glob_idx,
                               R=w.R, maxP=w.max_p, T=w.T, causal=w.causal, is_cross=w.cross)
        O.attn_fwd(qs, ks, vs, nb, va, scale=w.d ** -0.5, lowp=w.dtype == "bf16", fp32_w=False)
    dt = time.perf_counter() - t0
    desc = (f"{slices} of {w.B * w.n_kv} (batch, kv-group) slices ({rep} q heads x {w.N} queries "
            f"each) of {w.name}; full-job time extrapolated linearly in slices")
    return dt, desc, O.num_threads()


def cpu_baseline_value(w, dt, slices):
    full = dt * (w.B * w.n_kv) / slices
    return w.B * w.N / full, full


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def _plan(args, w, world):
    if args.shard != "auto":
        return args.shard if world > 1 else "single"
    if world == 1:
        return "single"
    return "rows" if w.B * w.n_kv < world or w.name == "c3" else "groups"


class _Job:
    """One rank's share of the workload's step: device tensors plus a
    step() that runs graph build + gather attention on them."""

    def __init__(self, plan, w, m, dev, world, rank):
        import torch
        from ssa_b200.sharding import GroupSharded, RowSharded
        from ssa_b200.workloads import make_x, project
        self.plan, self.w, self.m, self.world, self.rank = plan, w, m, world, rank
        self.causal = w.causal and not w.cross
        x, kv = make_x(w, dev, seed=1)           # the same job on every rank
        if plan == "rows":
            if w.cross or w.B != 1:
                raise SystemExit("query-row sharding is for one self-attention sequence (B=1)")
            self.runner = RowSharded(m, w.N, world, rank, causal=self.causal)
            r0, r1 = self.runner.rows
            xl = x[:, r0:r1]
            with torch.no_grad():
                self.q = m.Wq(xl).view(w.B, r1 - r0, w.H, w.d).transpose(1, 2)
                self.k_seq = m.Wk(xl).view(w.B, r1 - r0, w.n_kv, w.d).permute(1, 0, 2, 3).contiguous()
                self.v_seq = m.Wv(xl).view(w.B, r1 - r0, w.n_kv, w.d).permute(1, 0, 2, 3).contiguous()
            self.tokens_local = w.B * (r1 - r0)
        else:
            self.q, self.k, self.v = project(m, x, kv)
            if plan == "groups":
                self.runner = GroupSharded(m, world, rank, causal=w.causal, is_cross=w.cross)
                self.slices = self.runner.slices(w.B, w.n_kv)
                self.tokens_local = sum((s.b1 - s.b0) * (s.g1 - s.g0) for s in self.slices) * w.N // w.n_kv
            else:
                self.tokens_local = w.B * w.N
        del x, kv

    def step(self, stream, mark, mark_bwd=None):
        """Runs one step; records `mark` (a CUDA event) between the graph
        build and the attention where the plan has a single such point.
        With mark_bwd (training mode, single plan): the attention backward
        follows the forward, and mark_bwd is recorded between them."""
        import torch
        from ssa_b200 import ops
        m, w = self.m, self.w
        if self.plan == "single":
            nb, valid = m._graph(self.q, self.k, w.M, self.causal, w.cross)
            mark.record(stream)
            out, lse = ops.attn_fwd(self.q, self.k, self.v, nb, valid, m.scale, False,
                                    want_lse=mark_bwd is not None)
            if mark_bwd is not None:
                mark_bwd.record(stream)
                if getattr(self, "dO", None) is None:
                    self.dO = torch.ones_like(out)
                ops.attn_bwd(self.q, self.k, self.v, nb, valid, self.dO, lse, m.scale, False)
            return out
        if self.plan == "rows":
            from ssa_b200.sharding import gather_seq_major, seq_major_view
            k = seq_major_view(gather_seq_major(self.k_seq, self.runner.group))
            v_full, v_work = gather_seq_major(self.v_seq, self.runner.group, async_op=True)
            nb, valid = m._graph(self.q, k, w.N, self.causal, False, q_row0=self.runner.rows[0])
            mark.record(stream)
            v_work.wait()
            out, _ = ops.attn_fwd(self.q, k, seq_major_view(v_full), nb, valid, m.scale, False,
                                  want_lse=False)
            return out
        rep = w.H // w.n_kv
        from ssa_b200.sharding import slice_views
        graphs = []
        for s in self.slices:
            qs, ks, vs = slice_views(self.q, self.k, self.v, s, rep)
            graphs.append((qs, ks, vs) + tuple(m._graph(qs, ks, w.M, self.causal, w.cross)))
        mark.record(stream)
        return [ops.attn_fwd(qs, ks, vs, nb, valid, m.scale, False, want_lse=False)[0]
                for qs, ks, vs, nb, valid in graphs]


def workload_config(w) -> dict:
    """The `config` object of the JSON line: the workload alone, identical for
    both arms (how each arm runs it goes in top-level keys)."""
    return {"workload": w.name, "B": w.B, "N": w.N, "M": w.M, "H": w.H, "n_kv": w.n_kv,
            "d_head": w.d, "K": w.K, "window": w.window, "R": w.R, "probes": w.T,
            "causal": w.causal, "cross": w.cross}


def sample_stride(w, A: int) -> int:
    """Key-tile stride of the sample scan: the library's rule
    (graph_workspace_layout in ssa_graph.cu), restated for the FLOP count."""
    capg = ((6 * A + 64) + 7) // 8 * 8
    fit = capg * 8 // 272
    tiles = (w.M + 127) // 128
    s = max(A // 12, 1)
    if fit > 0 and -(-tiles // s) > fit:
        s = -(-tiles // fit)
    return s


def scan_flops(w, A: int):
    """Tensor-core FLOPs the two scan passes issue: per 128-row query tile,
    one 128 x 128 x d MMA per key tile visited (causal: tiles up to the
    tile's last row; the sample pass every s-th of them)."""
    tiles_all = (w.M + 127) // 128
    s = sample_stride(w, A)
    full = sample = 0
    for n0 in range(0, w.N, 128):
        n_hi = min(w.N, n0 + 128) - 1
        nkt = min(tiles_all, (n_hi >> 7) + 1) if (w.causal and not w.cross) else tiles_all
        full += nkt
        sample += -(-nkt // s)
    per = 2 * 128 * 128 * w.d * w.B * w.H
    return full * per, sample * per


def graph_roofline(w, m, stage_ms: dict, ms_graph: float, peaks: dict, traffic: dict):
    """Per-stage roofline of the graph build: the scans against the sustained
    bf16 tensor peak, every stage's measured DRAM bytes (ncu, profiles/) over
    its CUDA-event time against the HBM peak, and the build's compulsory bytes
    (q and k read, neighbors and valid written) over the whole build."""
    lsh = m.lsh_builder
    A = lsh.output_width(w.M, m.lsh_k)
    s = 4 if w.dtype == "fp32" else 2
    W = (2 * w.window + 1 if not w.cross else 0) + w.G + A
    W = min(w.K, W) if w.cross else min(w.K - 1, W) + 1
    hbm, tflops = peaks["hbm_gbs"], peaks["bf16_tflops_sustained"]
    out = {"peak_hbm_gbs": hbm, "peak_bf16_tflops_sustained": tflops, "stages": {}}
    full, sample = scan_flops(w, A)
    for name, ms in stage_ms.items():
        st = {"ms": round(ms, 4)}
        if ms > 0:
            if name in ("scan_full", "scan_sample") and w.dtype == "bf16":
                fl = full if name == "scan_full" else sample
                st.update({"bound": "tensor", "flops": fl, "tflops": fl / (ms / 1e3) / 1e12,
                           "frac": fl / (ms / 1e3) / 1e12 / tflops})
            tb = traffic.get(name)
            if tb:
                gbs = tb / (ms / 1e3) / 1e9
                st.update({"dram_bytes": tb, "dram_gbs": gbs, "dram_frac": gbs / hbm})
        out["stages"][name] = st
    comp = w.B * w.H * w.N * w.d * s + w.B * w.n_kv * w.M * w.d * s + w.B * w.H * w.N * W * 5
    out["compulsory_bytes"] = comp
    out["compulsory_gbs"] = comp / (ms_graph / 1e3) / 1e9
    out["compulsory_frac"] = out["compulsory_gbs"] / hbm
    dram = sum(traffic.get(n, 0) for n in stage_ms)
    out["dram_bytes_measured"] = dram or None
    return out


def time_job(job, stream, flush, steps, warmup, world, dev):
    """Warm-up, then `steps` timed steps of job (L2 flushed before each);
    returns the mean (step ms, graph-build ms), each the max over ranks."""
    import torch
    import torch.distributed as dist
    with torch.no_grad():
        for _ in range(max(warmup, 0)):
            flush.zero_()
            job.step(stream, torch.cuda.Event())
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        evs = []
        for _ in range(steps):
            flush.zero_()
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record(stream)
            job.step(stream, e1)
            e2.record(stream)
            evs.append((e0, e1, e2))
        torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(c) for a, b, c in evs)
    ms_graph = statistics.mean(a.elapsed_time(b) for a, b, c in evs)
    if world > 1:
        t = torch.tensor([ms, ms_graph], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_graph = [float(x) for x in t.tolist()]
    return ms, ms_graph


def time_captured(job, stream, flush, steps, warmup):
    """The same step (graph build + gather attention) captured once as a
    CUDA graph (ssa_b200.captured.CapturedStep) and replayed: for a
    launch-bound shape this removes the host side of a dozen launches.
    Returns its timing object, or the error if the capture fails."""
    import torch
    from ssa_b200.captured import CapturedStep
    w = job.w
    try:
        cs = CapturedStep(job.m, job.q, job.k, job.v, causal=job.causal, is_cross=w.cross)
        for _ in range(max(warmup, 0)):
            flush.zero_()
            cs()
        torch.cuda.synchronize()
        evs = []
        for _ in range(steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            cs()
            e1.record(stream)
            evs.append((e0, e1))
        torch.cuda.synchronize()
        ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
        del cs
        return {"value": w.B * w.N / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
                "note": "one CUDA graph replay per step (inputs already in the static buffers)"}
    except Exception as e:  # the eager figure above stands
        return {"error": f"{type(e).__name__}: {e}"[:300]}


def run_long_context(args, dev, flush, world, rank):
    """The long-context config c3 (B=1, N=32768) on the same GPUs: query-row
    sharding with the NCCL all-gather of K/V when world > 1, the whole job on
    one GPU otherwise. Returns its throughput object (rank 0) for the JSON
    line, so one run of bench.py --gpus N gives both scaling curves."""
    import torch
    from ssa_b200.workloads import WORKLOADS, make_module
    w = WORKLOADS["c3"]
    plan = "rows" if world > 1 else "single"
    m = make_module(w, dev)
    job = _Job(plan, w, m, dev, world, rank)
    ms, ms_graph = time_job(job, torch.cuda.current_stream(dev), flush, args.steps, args.warmup, world, dev)
    del job, m
    return {"workload": "c3", "value": w.B * w.N / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "graph_build_ms": ms_graph, "n_gpus": world, "scaling": "strong",
            "parallelism": ("query-row sharding: %d rows per GPU, K/V all-gathered (NCCL)" % (w.N // world)
                            if world > 1 else "one GPU, whole job"),
            "config": workload_config(w)}


def run_other_workloads(args, dev, flush, world, rank):
    """The other named configs on the same GPUs, fewer steps each: c1 and c5
    (graph build + gather attention; group sharding when world > 1) and, on
    one GPU, the c4 training step. One object per config, so one bench.py
    run records a throughput for every named shape."""
    import torch
    from ssa_b200.workloads import WORKLOADS, make_module
    steps, warmup = max(2, min(args.steps, 5)), max(3, min(args.warmup, 3))
    stream = torch.cuda.current_stream(dev)
    out = {}
    for name in ("c1", "c5"):
        w = WORKLOADS[name]
        plan = "single" if world == 1 else ("groups" if w.B * w.n_kv >= world else "rows")
        m = make_module(w, dev)
        job = _Job(plan, w, m, dev, world, rank)
        ms, ms_graph = time_job(job, stream, flush, steps, warmup, world, dev)
        out[name] = {"value": w.B * w.N / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
                     "graph_build_ms": ms_graph, "steps": steps, "warmup": warmup, "dtype": w.dtype,
                     "parallelism": "one GPU, whole job" if plan == "single" else
                     f"group sharding: {w.B * w.n_kv} (batch, kv-head) units over {world} GPUs",
                     "config": workload_config(w)}
        if name == "c1" and plan == "single":
            out[name]["graph_replay"] = time_captured(job, stream, flush, steps, warmup)
        del job, m
    if world == 1:
        w = WORKLOADS["c4"]
        res, _, _ = model_step_times(w, dev, steps, warmup, flush)
        out["c4"] = {"metric": "sparse-transformer training step (forward + out.sum().backward()) tokens/s",
                     "steps": steps, "warmup": warmup, "dtype": w.dtype,
                     "config": {**workload_config(w), "layers": w.layers, "vocab": w.vocab},
                     "models": res}
    return out


def model_step_times(w, dev, steps, warmup, flush, clocks=None):
    """Times the c4 model step of SparseTransformer and of
    CachedGraphSparseTransformer(reuse_every=4) on one GPU; returns
    ({model: times}, kernel launches of the first, its clock record)."""
    import torch
    from ssa_b200 import _lib
    from ssa_b200.attention import CachedGraphSparseTransformer, SparseTransformer
    cfg = w.config()
    torch.manual_seed(0)
    plain = SparseTransformer(cfg, num_layers=w.layers, vocab_size=w.vocab).to(dev)
    torch.manual_seed(0)
    embed = torch.nn.Embedding(w.vocab, w.d_model).to(dev)
    cached = CachedGraphSparseTransformer(cfg, num_layers=w.layers, reuse_every=4).to(dev)
    g = torch.Generator(device="cpu").manual_seed(1)
    ids = torch.randint(0, w.vocab, (w.B, w.N), generator=g).to(dev)

    def step_plain():
        out, _ = plain(ids)
        out.sum().backward()

    def step_cached():
        out, _ = cached(embed(ids))
        out.sum().backward()

    def fwd_only(fn):
        with torch.no_grad():
            fn()

    def timed(fn, steps):
        evs = []
        for _ in range(steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        return statistics.mean(x.elapsed_time(y) for x, y in evs)

    res = {}
    launches, clk = 0, None
    for name, fn, fwd in (("sparse_transformer", step_plain, lambda: plain(ids)),
                          ("cached_graph_transformer", step_cached, lambda: cached(embed(ids)))):
        for _ in range(max(warmup, 0)):
            fn()
        torch.cuda.synchronize()
        if name == "sparse_transformer":
            if clocks is not None:
                clocks.start()
            launches0 = _lib.load().ssa_kernel_launches()
        ms = timed(fn, steps)
        if name == "sparse_transformer":
            launches = _lib.load().ssa_kernel_launches() - launches0
            if clocks is not None:
                clk = clocks.stop()
        ms_fwd = timed(lambda: fwd_only(fwd), max(2, steps // 2))
        res[name] = {"value": w.B * w.N / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
                     "forward_ms": ms_fwd, "backward_ms": ms - ms_fwd}
        for p in list(plain.parameters()) + list(cached.parameters()) + list(embed.parameters()):
            p.grad = None
    return res, launches, clk


def run_model(args):
    """The training config's model step on one GPU: token ids -> embedding ->
    6 sparse-transformer layers -> out.sum().backward() (the reference's own
    training check, tests/test_gradients.py:17-18). SparseTransformer builds a
    graph in every layer; CachedGraphSparseTransformer(reuse_every=4) builds
    one per group of layers and reuses it (and its inverted index) in the
    group's forward and backward."""
    import torch
    from ssa_b200.workloads import WORKLOADS
    w = WORKLOADS[args.workload]
    if args.batch:
        w = type(w)(**{**w.__dict__, "B": args.batch})
    if not w.layers or w.layers < 2:
        raise SystemExit("--mode model is for the training config (c4)")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    res, launches, clk = model_step_times(w, dev, args.steps, args.warmup, flush, ClockSampler(0))
    main = res["sparse_transformer"]
    out = {"metric": "sparse-transformer training step (forward + out.sum().backward()) tokens/s",
           "value": main["value"], "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": main["ms_per_step"], "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": w.dtype,
           "data": "synthetic (uniform random token ids; random-init weights in reference order)",
           "config": {**workload_config(w), "layers": w.layers, "vocab": w.vocab},
           "parallelism": "one GPU, whole job", "l2": "flushed (256 MB write) between timed steps",
           "models": res, "gpu_launches": launches, "clocks": clk}
    print(json.dumps(out))
    return out


def run_gpu(args):
    import torch
    import torch.distributed as dist

    from ssa_b200 import _lib
    from ssa_b200.workloads import WORKLOADS, make_module

    world, rank, local = dist_info()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    w = WORKLOADS[args.workload]
    if args.batch:
        w = type(w)(**{**w.__dict__, "B": args.batch})
    plan = _plan(args, w, world)
    if args.mode == "train" and plan != "single":
        raise SystemExit("--mode train runs on one GPU (one layer's attention core)")
    m = make_module(w, dev)
    job = _Job(plan, w, m, dev, world, rank)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    with torch.no_grad():
        train = args.mode == "train"
        for _ in range(max(args.warmup, 0)):
            flush.zero_()
            job.step(stream, torch.cuda.Event(), torch.cuda.Event() if train else None)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        clocks = ClockSampler(local)
        clocks.start()
        torch.cuda.synchronize()
        launches0 = _lib.load().ssa_kernel_launches()
        evs = []
        for _ in range(args.steps):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e2 = torch.cuda.Event(enable_timing=True)
            eb = torch.cuda.Event(enable_timing=True) if train else None
            e0.record(stream)
            job.step(stream, e1, eb)
            e2.record(stream)
            evs.append((e0, e1, e2, eb))
        torch.cuda.synchronize()
        launches = _lib.load().ssa_kernel_launches() - launches0
        if world > 1:
            dist.barrier()
        clk = clocks.stop()
    tot = [a.elapsed_time(c) for a, b, c, _ in evs]
    graph = [a.elapsed_time(b) for a, b, c, _ in evs]
    attn = [b.elapsed_time(eb if eb is not None else c) for a, b, c, eb in evs]
    bwd = [eb.elapsed_time(c) for a, b, c, eb in evs if eb is not None]
    ms = statistics.mean(tot)
    ms_graph, ms_attn = statistics.mean(graph), statistics.mean(attn)
    ms_bwd = statistics.mean(bwd) if bwd else None
    launches_all = launches
    if world > 1:
        t = torch.tensor([ms, ms_graph, ms_attn], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_graph, ms_attn = [float(x) for x in t.tolist()]
        c = torch.tensor([launches], device=dev, dtype=torch.float64)
        dist.all_reduce(c)
        launches_all = int(c.item())

    tokens = w.B * w.N                      # the whole job, split over the ranks
    value = tokens / (ms / 1e3)
    peak, peak_src = hbm_peak()
    alg_bytes = w.bytes_per_token() * job.tokens_local   # this rank's attention bytes
    attn_gbs = alg_bytes / (ms_attn / 1e3) / 1e9
    step_gbs = w.bytes_per_token() * tokens / (ms / 1e3) / 1e9 / world
    traffic, graph_traffic = None, {}
    try:
        with open(TRAFFIC_FILE) as f:
            tw = json.load(f).get(w.name, {})
        if plan == "single" and tw.get("batch") == w.B:
            traffic = tw.get("k_attn_fwd")
            graph_traffic = tw.get("graph", {})
    except Exception:
        pass

    # Per-stage times of the graph build: CUDA events the library records at
    # its stage boundaries (ssa_graph_profile), on extra steps after the timed
    # ones, L2 flushed before each.
    stage_ms = None
    if plan == "single" and not args.no_graph_profile:
        from ssa_b200 import ops
        samples = []
        with torch.no_grad(), ops.graph_profile() as prof:
            for _ in range(3):
                flush.zero_()
                m._graph(job.q, job.k, w.M, job.causal, w.cross)
                samples.append(prof.times())
        stage_ms = {k: statistics.median(x[k] for x in samples) for k in samples[0]}

    # End to end through the public API with host buffers: pinned q/k/v in,
    # attention output back to pinned host memory, copies inside the timing.
    e2e = None
    if not args.no_e2e and args.mode == "fwd":
        e2e = run_e2e(args, job, dev, flush, world)

    # The long-context config on the same GPUs, as a second object; then the
    # other named configs.
    long_ctx, others = None, None
    if args.workload == "c2" and args.mode == "fwd" and not args.batch and not args.no_long_context:
        long_ctx = run_long_context(args, dev, flush, world, rank)
    if args.workload == "c2" and args.mode == "fwd" and not args.batch and not args.no_other_workloads:
        others = run_other_workloads(args, dev, flush, world, rank)

    result = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1 and args.mode == "fwd":
            dt, desc, cores = cpu_sample(w, m, job.q, job.k, job.v, args.baseline_slices)
            val, _full = cpu_baseline_value(w, dt, args.baseline_slices)
            cpu = {"value": val, "unit": "tokens/s", "cores": cores, "kind": "port",
                   "sample": desc, "sample_seconds": round(dt, 3)}
        par = {"single": "one GPU, whole job",
               "groups": f"group sharding: {w.B * w.n_kv} (batch, kv-head) units over {world} GPUs, no collective",
               "rows": f"query-row sharding: {w.N // world} rows per GPU, K/V all-gathered (NCCL)"}[plan]
        metric = METRIC if args.mode == "fwd" else \
            "sparse-attn train step (graph + attention fwd + bwd) tokens/s/GPU, one layer's attention core"
        attn_dram = None
        if traffic:
            g_ = traffic / (ms_attn / 1e3) / 1e9
            attn_dram = {"dram_gbs": g_, "dram_frac": g_ / peak}
        result = {
            "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": w.dtype,
            "data": "synthetic (seeded N(0,1) activations; random-init weights in reference order)",
            "config": workload_config(w),
            "parallelism": par,
            "l2": "flushed (256 MB write) between timed steps",
            "roofline": {"kernel": "k_attn_fwd", "bound": "hbm", "achieved": attn_gbs, "peak": peak,
                         "unit": "GB/s", "frac": attn_gbs / peak, "traffic": traffic,
                         "peak_source": f"{peak_src} hbm_gbs",
                         "algorithmic_bytes": alg_bytes,
                         **(attn_dram or {}),
                         "note": "achieved counts algorithmic bytes (gathered K/V rows + q + out); the "
                                 "GQA heads of a kv group re-gather the same rows from L2, so it can "
                                 "exceed the HBM peak; dram_frac is the measured DRAM traffic"},
            "step_roofline": {"achieved": step_gbs, "frac": step_gbs / peak, "unit": "GB/s",
                              "note": "attention algorithmic bytes over graph build + attention, per GPU"},
            "graph_roofline": (graph_roofline(w, m, stage_ms, ms_graph, peaks(), graph_traffic)
                               if stage_ms else None),
            "kernels_ms": {"graph_build": ms_graph, "attention": ms_attn,
                           "graph_build_per_step": [round(x, 3) for x in graph],
                           **({"graph_stages": {k: round(v, 4) for k, v in stage_ms.items()}} if stage_ms else {}),
                           **({"attention_backward": ms_bwd} if ms_bwd is not None else {})},
            "gpu_launches": launches_all,
            "clocks": clk,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "long_context": long_ctx,
            "other_workloads": others,
        }
        print(json.dumps(result))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def e2e_spans(slices, target):
    """Pipeline chunks of the end-to-end step as (batch, kv0, kv1) spans of
    one batch element each: the rank's slices per batch element, halved
    (all together) while there are fewer than `target` chunks and every
    span keeps at least two kv heads; then one kv head is split off the
    front of the first chunk and off the back of the last one, since only
    the first copy-in and the last copy-out overlap no compute."""
    spans = [(b, s.g0, s.g1) for s in slices for b in range(s.b0, s.b1)]
    while len(spans) < target and all((g1 - g0) % 2 == 0 and g1 - g0 >= 4 for _, g0, g1 in spans):
        spans = [(b, g, g + (g1 - g0) // 2) for b, g0, g1 in spans for g in (g0, g0 + (g1 - g0) // 2)]
    if spans and spans[0][2] - spans[0][1] > 1:
        b, g0, g1 = spans[0]
        spans[0:1] = [(b, g0, g0 + 1), (b, g0 + 1, g1)]
    if spans and spans[-1][2] - spans[-1][1] > 1:
        b, g0, g1 = spans[-1]
        spans[-1:] = [(b, g0, g1 - 1), (b, g1 - 1, g1)]
    return spans


def run_e2e(args, job, dev, flush, world):
    """The same step through the public API from pinned host memory: this
    rank's inputs copied in, its outputs copied back, inside the timing.
    The step is cut into chunks (e2e_spans: kv-head ranges of one batch
    element); chunk i+1 is copied in on one stream while chunk i computes,
    and results go back on a third stream, so PCIe transfers overlap the
    kernels."""
    import torch
    import torch.distributed as dist
    from ssa_b200.sharding import GroupSlice, slice_views
    w, m = job.w, job.m
    stream = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)

    def pin(t):
        return t.detach().contiguous().cpu().pin_memory()

    rep = w.H // w.n_kv
    if job.plan == "rows":
        chunks = [(pin(job.q.transpose(1, 2)), pin(job.k_seq), pin(job.v_seq))]   # (B,n,H,d), (m,B,n_kv,d)
    else:
        slices = job.slices if job.plan == "groups" else [GroupSlice(0, w.B, 0, w.n_kv)]
        views = [slice_views(job.q, job.k, job.v, GroupSlice(b, b + 1, g0, g1), rep)
                 for b, g0, g1 in e2e_spans(slices, args.e2e_chunks)]
        chunks = [tuple(pin(t.transpose(1, 2)) for t in vw) for vw in views]      # (b, N|M, heads, d)
    outs_h = [torch.empty((c[0].shape[0], c[0].shape[1], w.H if job.plan == "rows" else c[0].shape[2], w.d),
                          dtype=job.q.dtype).pin_memory() for c in chunks]
    devs = [[torch.empty_like(h, device=dev) for h in c] for c in chunks]

    def compute(i):
        dq_, dk_, dv_ = devs[i]
        if job.plan == "rows":
            return job.runner.step(dq_.transpose(1, 2), dk_, dv_)
        q4, k4, v4 = dq_.transpose(1, 2), dk_.transpose(1, 2), dv_.transpose(1, 2)
        nb, valid = m.build_graph(q4, k4, w.N, w.M, q4.shape[0], dev, job.causal, w.cross)
        return m.apply_graph(q4, k4, v4, nb, valid)

    def one():
        s_in.wait_stream(stream)
        ev_in = []
        for c, d_ in zip(chunks, devs):
            with torch.cuda.stream(s_in):
                for dt, ht in zip(d_, c):
                    dt.copy_(ht, non_blocking=True)
            e = torch.cuda.Event()
            e.record(s_in)
            ev_in.append(e)
        for i in range(len(chunks)):
            stream.wait_event(ev_in[i])
            out = compute(i)
            e = torch.cuda.Event()
            e.record(stream)
            s_out.wait_event(e)
            with torch.cuda.stream(s_out):
                outs_h[i].copy_(out.transpose(1, 2), non_blocking=True)
            out.record_stream(s_out)
        stream.wait_stream(s_out)

    with torch.no_grad():
        for _ in range(max(1, args.warmup)):
            one()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        evs = []
        for _ in range(args.steps):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            one()
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize()
    ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    h2d = sum(h.numel() * h.element_size() for c in chunks for h in c)
    d2h = sum(o.numel() * o.element_size() for o in outs_h)
    if world > 1:
        t = torch.tensor([ms, float(h2d), float(d2h)], device=dev, dtype=torch.float64)
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(t)
        ms, h2d, d2h = float(mx[0]), int(t[1]), int(t[2])
    api = ("RowSharded.step (NCCL all-gather of K/V + graph + attention)" if job.plan == "rows"
           else "SparseAttention.build_graph + apply_graph (int64/bool graph contract)")
    return {"value": w.B * w.N / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "api": api,
            "chunks": len(chunks), "overlap": "H2D, compute and D2H on three streams, per chunk"}


# ---------------------------------------------------------------------------
# Reference arm: the CPU restatement (oracle port) on the host cores
# ---------------------------------------------------------------------------
def run_reference(args):
    world, rank, local = dist_info()
    if rank != 0:
        return None
    import torch
    from ssa_b200.workloads import WORKLOADS, make_module, make_x, project

    w = WORKLOADS[args.workload]
    torch.set_num_threads(os.cpu_count() or 1)
    m = make_module(w, "cpu")
    slices = args.baseline_slices
    ng = min(slices, w.n_kv)                 # kv groups in the sample (batch row 0)
    rep = w.H // w.n_kv
    x, kv = make_x(w, "cpu", seed=1, batch=1)
    src = kv if kv is not None else x
    with torch.no_grad():                     # project only the sampled heads' columns
        def proj(lin, rows_, inp, heads):
            y = inp.float() @ lin.weight[:rows_].float().T
            return y.to(w.torch_dtype).view(1, inp.shape[1], heads, w.d).transpose(1, 2)
        q = proj(m.Wq, ng * rep * w.d, x, ng * rep)
        k = proj(m.Wk, ng * w.d, src, ng)
        v = proj(m.Wv, ng * w.d, src, ng)
    del x, kv, src
    w1 = type(w)(**{**w.__dict__, "B": 1, "H": ng * rep, "n_kv": ng,
                    "d_model": ng * rep * w.d})
    slices = min(slices, ng)
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_sample(w1, m, q, k, v, 1)
    times = []
    desc, cores = "", 1
    for _ in range(args.steps):
        dt, desc, cores = cpu_sample(w1, m, q, k, v, slices)
        times.append(dt)
    dt = statistics.mean(times)
    factor = (w.B * w.n_kv) / slices
    full = dt * factor
    value = w.B * w.N / full
    desc = desc.replace(f"{slices} of {w1.B * w1.n_kv}", f"{slices} of {w.B * w.n_kv}")
    res = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": dt * 1e3,
           "extrapolation": {"factor": factor, "full_job_ms": full * 1e3,
                             "note": "each step times the sample; value = the whole job's tokens over "
                                     "the sample time x factor (linear in (batch, kv-group) slices)"},
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": w.dtype,
           "data": "synthetic", "config": workload_config(w),
           "parallelism": f"reference arm: the CPU oracle port on {cores} host threads, rank 0 only",
           "l2": "n/a (CPU arm)",
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                            "sample": desc},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(res))
    return res


def run_proj(args):
    """QKV projection + graph build from the activations x, one GPU: the
    fused tcgen05 projection whose epilogue hashes q and k
    (ssa_qkv_proj_hash, then ssa_build_graph_prehashed) against torch
    Linear (cuBLAS) + ssa_build_graph. Self-attention bf16 configs."""
    import torch
    from ssa_b200 import _lib, ops
    from ssa_b200.workloads import WORKLOADS, make_module, make_x
    w = WORKLOADS[args.workload]
    if args.batch:
        w = type(w)(**{**w.__dict__, "B": args.batch})
    if w.cross or w.dtype != "bf16":
        raise SystemExit("--mode proj is for bf16 self-attention configs (c2, c3)")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    m = make_module(w, dev)
    x, _ = make_x(w, dev, seed=1)
    W = torch.cat([m.Wq.weight, m.Wk.weight, m.Wv.weight]).detach()
    lsh = m.lsh_builder
    kw = dict(H=w.H, n_kv=w.n_kv, R=lsh.R, max_p=lsh.max_P, p_eff=lsh.compute_effective_p(w.N, lsh.C, lsh.max_P),
              C=lsh.C, T=lsh.T, A=lsh.output_width(w.N, m.lsh_k), causal=w.causal, K=m.K, window=w.window)
    glob = m._glob(w.N, dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def fused():
        qkv, st = ops.qkv_project_hash(x, W, lsh.rand_proj, glob, **kw)
        q, k, _ = ops.split_qkv(qkv, w.H, w.n_kv)
        return ops.build_graph_prehashed(q, k, st)

    def unfused():
        qkv = torch.nn.functional.linear(x, W)
        q, k, _ = ops.split_qkv(qkv, w.H, w.n_kv)
        return m._graph(q, k, w.M, w.causal, False)

    def timed(fn):
        for _ in range(max(args.warmup, 0)):
            fn()
        torch.cuda.synchronize()
        evs = []
        for _ in range(args.steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        return statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)

    with torch.no_grad():
        if ops.qkv_project_hash(x, W, lsh.rand_proj, glob, **kw) is None:
            raise SystemExit("the fused projection does not serve this config")
        clocks = ClockSampler(0)
        clocks.start()
        launches0 = _lib.load().ssa_kernel_launches()
        ms_f = timed(fused)
        launches = (_lib.load().ssa_kernel_launches() - launches0) // max(args.steps + max(args.warmup, 0), 1)
        ms_u = timed(unfused)
        clk = clocks.stop()
        nb_f, va_f = fused()
        nb_u, va_u = unfused()
        same = bool(torch.equal(va_f, va_u) and torch.equal(nb_f[va_u.bool()], nb_u[va_u.bool()]))
    tokens = w.B * w.N
    out = {"metric": "QKV projection + graph build tokens/s (fused tcgen05 projection + hash epilogue)",
           "value": tokens / (ms_f / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": ms_f, "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (seeded activations; random-init weights in reference order)",
           "config": {**workload_config(w), "d_model": w.d_model},
           "parallelism": "one GPU, whole job", "l2": "flushed (256 MB write) between timed steps",
           "unfused_ms_per_step": ms_u, "unfused": "torch Linear (cuBLAS) + ssa_build_graph",
           "graphs_equal": same, "gpu_launches_per_step": launches, "clocks": clk}
    print(json.dumps(out))
    return out


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "model":
        run_model(args)
    elif args.mode == "proj":
        run_proj(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
