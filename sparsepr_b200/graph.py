"""CUDA-graph capture of one SparsePR attention layer.

Every step of ``sparse_attention`` is stream-ordered device work with no host
synchronisation (fixed-density budgets), so a whole layer — role factors,
both k-means runs, permutes, scores, selection, block-sparse attention, dense
probes, fit and repair — can be captured once and replayed with a single
launch.  Inputs are copied into static device buffers before each replay.
"""

from __future__ import annotations

import torch

from .attention import sparse_attention
from .n8_v6 import N8V6Config, N8V6Core

__all__ = ["GraphedSparseAttention"]


class GraphedSparseAttention:
    """Captured cold-start SparsePR layer for fixed ``[B,H,N,D]`` bf16 inputs.

    Each replay routes from scratch (a fresh core per call, like the first
    denoising step), so replays are independent of each other.
    ``selector_budget_mode`` must be ``fixed_density`` (the top-p mode reads
    its density on the host).
    """

    def __init__(self, shape, config: N8V6Config, device: torch.device, warmup: int = 2):
        if config.selector_budget_mode != "fixed_density":
            raise ValueError("graph capture needs selector_budget_mode='fixed_density'")
        self.config = config
        self.device = device
        self.q = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.k = torch.zeros_like(self.q)
        self.v = torch.zeros_like(self.q)
        self.graph = None
        self._warmup = warmup

    def _run(self):
        return sparse_attention(self.q, self.k, self.v, N8V6Core(self.config))

    def capture(self):
        """Warm up on a side stream (caches workspaces and index constants), then capture."""
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(self._warmup):
                self._run()
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out, self.density, self.info = self._run()
        return self

    def load(self, q, k, v):
        """Copy inputs (device or pinned host tensors) into the static buffers."""
        self.q.copy_(q, non_blocking=True)
        self.k.copy_(k, non_blocking=True)
        self.v.copy_(v, non_blocking=True)

    def replay(self):
        if self.graph is None:
            self.capture()
        self.graph.replay()
        return self.out

    def __call__(self, q, k, v):
        self.load(q, k, v)
        return self.replay()
