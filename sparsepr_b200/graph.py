"""CUDA-graph capture of one SparsePR attention layer, and a host-buffer front
end that streams a layer through captured graphs in head chunks.

Every step of ``sparse_attention`` is stream-ordered device work with no host
synchronisation (the top-p budget density stays on the device), so a whole layer — role factors,
both k-means runs, permutes, scores, selection, block-sparse attention, dense
probes, fit and repair — can be captured once and replayed with a single
launch.  Inputs are copied into static device buffers before each replay.
"""

from __future__ import annotations

import itertools

import torch

from . import kernels as K
from .attention import sparse_attention
from .n8_v6 import N8V6Config, N8V6Core
from .synthetic import random_init_indices

__all__ = ["GraphedSparseAttention", "StreamedSparseAttention", "ConcurrentSparseAttention"]

_SCOPE_IDS = itertools.count()


class GraphedSparseAttention:
    """Captured cold-start SparsePR layer for fixed ``[B,H,N,D]`` bf16 inputs.

    Each replay routes from scratch (a fresh core per call, like the first
    denoising step), so replays are independent of each other.
    With ``svg_ear_top_p`` budgets ``density`` is a 0-dim device tensor
    updated by every replay.  The graph's kernels use workspaces private to
    this object, so different graphs may replay concurrently on different
    streams.
    """

    def __init__(self, shape, config: N8V6Config, device: torch.device, warmup: int = 2, inputs=None):
        """``inputs`` (optional): three device bf16 tensors of ``shape`` to use as
        the static input buffers instead of private ones (e.g. views of a larger
        buffer shared by several graphs)."""
        self.config = config
        self.device = device
        if inputs is None:
            self.q = torch.zeros(shape, dtype=torch.bfloat16, device=device)
            self.k = torch.zeros_like(self.q)
            self.v = torch.zeros_like(self.q)
        else:
            self.q, self.k, self.v = inputs
            if any(tuple(t.shape) != tuple(shape) or t.dtype != torch.bfloat16 or not t.is_contiguous()
                   for t in inputs):
                raise ValueError(f"graph inputs must be contiguous bf16 tensors of shape {tuple(shape)}")
        self.graph = None
        self._warmup = warmup
        self._scope = f"graph{next(_SCOPE_IDS)}"
        # Cold-start centroid rows: a static input of the graph (default: the
        # config's own draw for this batch; load(..., init_rows) selects others).
        b, h, n, _d = shape
        self.k_init = random_init_indices(b * h, n, config.num_k_centroids, config.kmeans_init_seed).to(device)
        self.q_init = random_init_indices(b * h, n, config.num_q_centroids, config.kmeans_init_seed + 1).to(device)

    def init_rows(self, offset: int, total: int):
        """Device copies of rows ``[offset, offset + BH)`` of the cold-start draw
        for ``total`` problems (pass them to ``load``)."""
        bh = self.k_init.shape[0]
        n = self.q.shape[2]
        cfg = self.config
        k = random_init_indices(total, n, cfg.num_k_centroids, cfg.kmeans_init_seed)[offset:offset + bh]
        q = random_init_indices(total, n, cfg.num_q_centroids, cfg.kmeans_init_seed + 1)[offset:offset + bh]
        return k.to(self.device), q.to(self.device)

    def _run(self):
        with K.workspace_scope(self._scope):
            core = N8V6Core(self.config, init_indices=(self.k_init, self.q_init))
            return sparse_attention(self.q, self.k, self.v, core)

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

    def load(self, q, k, v, init_rows=None):
        """Copy inputs (device or pinned host tensors) into the static buffers;
        ``init_rows`` = a pair from ``init_rows()`` (device tensors)."""
        self.q.copy_(q, non_blocking=True)
        self.k.copy_(k, non_blocking=True)
        self.v.copy_(v, non_blocking=True)
        if init_rows is not None:
            self.k_init.copy_(init_rows[0], non_blocking=True)
            self.q_init.copy_(init_rows[1], non_blocking=True)

    def replay(self):
        if self.graph is None:
            self.capture()
        self.graph.replay()
        return self.out

    def __call__(self, q, k, v):
        self.load(q, k, v)
        return self.replay()


class StreamedSparseAttention:
    """SparsePR layer on host tensors, streamed through captured graphs by head chunks.

    ``__call__(hq, hk, hv, hout)`` takes pinned host ``[B,H,N,D]`` bf16
    tensors and writes the repaired output into the pinned host ``hout``.
    Heads are independent in every step of the layer, so the heads are cut
    into chunks of ``heads_per_chunk``; chunk i's host-to-device copy, graph
    replay and device-to-host copy are queued on stream ``i % slots``.  The
    copy engines then move one chunk while the SMs compute another.  Each
    chunk starts its k-means from its rows of the all-heads cold-start draw,
    and no step of the layer mixes heads, so the result equals one
    ``GraphedSparseAttention`` call over all heads.
    """

    def __init__(self, shape, config: N8V6Config, device: torch.device, heads_per_chunk: int = 8,
                 slots: int = 2, warmup: int = 2):
        b, h, n, d = shape
        if h % heads_per_chunk:
            raise ValueError(f"{h} heads do not split into chunks of {heads_per_chunk}")
        if b != 1:
            raise ValueError("streamed layers take B=1 (one [H,N,D] problem set per call)")
        self.shape = tuple(shape)
        self.device = device
        self.chunks = [(h0, h0 + heads_per_chunk) for h0 in range(0, h, heads_per_chunk)]
        nslots = min(slots, len(self.chunks))
        self.slots = [GraphedSparseAttention((b, heads_per_chunk, n, d), config, device, warmup)
                      for _ in range(nslots)]
        self.streams = [torch.cuda.Stream(device) for _ in range(nslots)]
        # Each chunk's rows of the all-heads cold-start draw (device, loaded per replay).
        self.init = [self.slots[0].init_rows(h0, h) for h0, _h1 in self.chunks]

    def capture(self):
        for g in self.slots:
            g.capture()
        return self

    def __call__(self, hq, hk, hv, hout):
        if any(g.graph is None for g in self.slots):
            self.capture()
        cur = torch.cuda.current_stream(self.device)
        for st in self.streams:
            st.wait_stream(cur)
        for i, (h0, h1) in enumerate(self.chunks):
            g = self.slots[i % len(self.slots)]
            with torch.cuda.stream(self.streams[i % len(self.slots)]):
                g.load(hq[:, h0:h1], hk[:, h0:h1], hv[:, h0:h1], self.init[i])
                g.graph.replay()
                hout[:, h0:h1].copy_(g.out, non_blocking=True)
        for st in self.streams:
            cur.wait_stream(st)
        return hout


class ConcurrentSparseAttention:
    """One SparsePR layer on device-resident ``[1,H,N,D]`` bf16 inputs, run as
    ``chunks`` captured graphs over contiguous head ranges, replayed
    concurrently on their own streams.

    Heads are independent in every step of the layer, but several steps are
    latency-bound and occupy few SMs (the Jacobi eigensolver runs one CTA per
    head; the small per-head linear algebra and the sort kernels are short).
    Two head chains replayed together let some of one chain's latency-bound
    kernels run beside the other chain's; the attention kernel itself holds an
    SM's whole shared memory and tensor memory, so nothing runs beside it
    (staggering the chains so one routes while the other attends was measured
    and serialised completely).  The graphs read views of
    one set of static input buffers (``load`` copies the inputs once) and each
    starts its k-means from its rows of the all-heads cold-start draw, so the
    outputs equal one all-heads call.  ``replay()`` returns the per-chunk
    outputs (head ranges in order); ``output()`` concatenates them.
    """

    def __init__(self, shape, config: N8V6Config, device: torch.device, chunks: int = 2, warmup: int = 2,
                 head_offset: int = 0, total_heads: int | None = None):
        """``head_offset`` / ``total_heads``: these heads are rows
        ``[head_offset, head_offset + H)`` of a ``total_heads``-head layer (a
        rank's shard); the cold-start draw is that layer's."""
        b, h, n, d = shape
        total = h if total_heads is None else int(total_heads)
        if b != 1:
            raise ValueError("concurrent layers take B=1")
        chunks = max(1, min(int(chunks), h))
        bounds = [h * i // chunks for i in range(chunks + 1)]
        self.ranges = [(bounds[i], bounds[i + 1]) for i in range(chunks) if bounds[i + 1] > bounds[i]]
        self.device = device
        self.q = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.k = torch.zeros_like(self.q)
        self.v = torch.zeros_like(self.q)
        self.graphs = []
        for h0, h1 in self.ranges:
            g = GraphedSparseAttention((1, h1 - h0, n, d), config, device, warmup,
                                       inputs=(self.q[:, h0:h1], self.k[:, h0:h1], self.v[:, h0:h1]))
            rows = g.init_rows(head_offset + h0, total)
            g.k_init.copy_(rows[0])
            g.q_init.copy_(rows[1])
            self.graphs.append(g)
        self.streams = [torch.cuda.Stream(device) for _ in self.graphs]

    def capture(self):
        for g in self.graphs:
            g.capture()
        return self

    def load(self, q, k, v):
        self.q.copy_(q, non_blocking=True)
        self.k.copy_(k, non_blocking=True)
        self.v.copy_(v, non_blocking=True)

    def replay(self):
        if any(g.graph is None for g in self.graphs):
            self.capture()
        cur = torch.cuda.current_stream(self.device)
        for st in self.streams:
            st.wait_stream(cur)
        for g, st in zip(self.graphs, self.streams):
            with torch.cuda.stream(st):
                g.graph.replay()
        for st in self.streams:
            cur.wait_stream(st)
        return [g.out for g in self.graphs]

    def output(self):
        """All heads' repaired output, ``[1,H,N,D]`` (a copy)."""
        return torch.cat([g.out for g in self.graphs], dim=1)

    def __call__(self, q, k, v):
        self.load(q, k, v)
        self.replay()
        return self.output()
