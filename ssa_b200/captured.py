"""Graph build + gather attention captured once as a CUDA graph and replayed.

`SparseAttention` in eval mode runs, per call, about a dozen kernels of this
package (hash, bucket trim, candidate scans, row stages, exact fallback,
gather attention), each behind a ctypes call and a few tensor allocations.
For small shapes the host side of that sequence, not the GPU, sets the step
time. `CapturedStep` records the sequence for fixed shapes once -- inputs
in static buffers, workspaces and outputs in the graph's private memory
pool -- and each call then copies new inputs in (if given) and launches
the whole step as one graph. The kernels and their arguments are the ones
the eager path launches, so the outputs are bit-identical to it.

Reference counterpart: `SparseAttention.build_graph` + `apply_graph`
(sparse_attention.py:1325-1418) for one fixed (q, k, v) shape.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops


class CapturedStep:
    """One captured eval step of `module` (a SparseAttention) on q (B,H,N,d)
    and k, v (B,n_kv,M,d) of fixed shapes, dtypes and strides.

    module: the SparseAttention whose hyperplanes, globals and config the
        step uses (read at capture time; later changes to them are not seen).
    causal / is_cross: as `module.build_graph`; by default the module's
        causal setting for self-attention.
    """

    def __init__(self, module, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                 causal: Optional[bool] = None, is_cross: bool = False, warmup: int = 2):
        if not (q.is_cuda and k.is_cuda and v.is_cuda):
            raise RuntimeError("CapturedStep needs CUDA tensors")
        self.module = module
        self.is_cross = bool(is_cross)
        base = module.config.causal if causal is None else bool(causal)
        self.causal = base and not self.is_cross
        self.M = k.shape[2]
        # Static inputs with the callers' strides (clone keeps a dense
        # permuted layout), so the captured kernels see the same layout.
        self.q, self.k, self.v = q.clone(), k.clone(), v.clone()
        dev = q.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.no_grad(), torch.cuda.stream(side):
            for _ in range(max(1, warmup)):  # library set-up (function attributes, tensor maps) before capture
                self._step()
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            self.out = self._step()

    def _step(self) -> torch.Tensor:
        m = self.module
        nb, valid = m._graph(self.q, self.k, self.M, self.causal, self.is_cross)
        out, _ = ops.attn_fwd(self.q, self.k, self.v, nb, valid, m.scale, m.config.fp32_attn_weights,
                              want_lse=False)
        return out

    def __call__(self, q: Optional[torch.Tensor] = None, k: Optional[torch.Tensor] = None,
                 v: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Copies the given inputs into the static buffers (same shapes and
        dtypes as at capture) and replays the step on the current stream.
        Returns the static output buffer (B,H,N,d), overwritten by the next
        call: clone it to keep it."""
        for src, dst in ((q, self.q), (k, self.k), (v, self.v)):
            if src is not None:
                if src.shape != dst.shape or src.dtype != dst.dtype:
                    raise ValueError(f"CapturedStep: input {tuple(src.shape)} {src.dtype} does not match the "
                                     f"captured {tuple(dst.shape)} {dst.dtype}")
                dst.copy_(src)
        self.graph.replay()
        return self.out
