"""Sequence-sharded front end for the SparsePR layer (Ulysses-style exchange).

When a model runs sequence-parallel, each of W ranks holds a contiguous slice
of the tokens for every head (``[B, N/W, H, D]``, BLHD).  SparsePR routes each
head over all of its tokens, so one all-to-all regroups the activations into
head shards (``[B, H/W, N, D]``, BHLD: all tokens of H/W heads), the layer runs
on the local heads with no further communication, and a second all-to-all
returns the output to sequence shards.  Each tensor crosses the fabric once per
direction: (W-1)/W of it, i.e. about 85 MB per tensor per GPU at config 3 with
W = 8.  With NCCL the exchange runs over NVLink / NVSwitch; the received data
lands in local HBM before any kernel reads it.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["seq_to_head", "head_to_seq", "UlyssesSparseAttention"]


def _world(group):
    return dist.get_world_size(group)


def seq_to_head(x: torch.Tensor, group=None) -> torch.Tensor:
    """``[B, N/W, H, D]`` sequence shard -> ``[B, H/W, N, D]`` head shard (all tokens).

    Rank r receives heads ``[r*H/W, (r+1)*H/W)``; tokens come back in rank
    order, so the sequence order is the global one."""
    w = _world(group)
    b, ns, h, d = x.shape
    if h % w:
        raise ValueError(f"{h} heads do not split over {w} ranks")
    hs = h // w
    send = x.reshape(b, ns, w, hs, d).permute(2, 0, 1, 3, 4).contiguous()  # [W(dest), B, Ns, Hs, D]
    recv = torch.empty_like(send)                                           # [W(src),  B, Ns, Hs, D]
    dist.all_to_all_single(recv, send, group=group)
    return recv.permute(1, 3, 0, 2, 4).reshape(b, hs, w * ns, d)


def head_to_seq(o: torch.Tensor, group=None) -> torch.Tensor:
    """Inverse of :func:`seq_to_head`: ``[B, H/W, N, D]`` -> ``[B, N/W, H, D]``."""
    w = _world(group)
    b, hs, n, d = o.shape
    if n % w:
        raise ValueError(f"{n} tokens do not split over {w} ranks")
    ns = n // w
    send = o.reshape(b, hs, w, ns, d).permute(2, 0, 3, 1, 4).contiguous()  # [W(dest), B, Ns, Hs, D]
    recv = torch.empty_like(send)                                          # [W(src),  B, Ns, Hs, D]
    dist.all_to_all_single(recv, send, group=group)
    return recv.permute(1, 2, 0, 3, 4).reshape(b, ns, w * hs, d)


class UlyssesSparseAttention:
    """SparsePR layer on sequence-sharded ``[B, N/W, H, D]`` q, k, v.

    ``attention(q, k, v) -> out`` is the head-local layer on ``[B, H/W, N, D]``
    tensors (default: ``sparse_attention`` with one ``N8V6Core`` per rank, which
    owns this rank's heads and their cross-step state).  Returns the output in
    the caller's sequence-sharded layout."""

    def __init__(self, config=None, group=None, attention=None):
        self.group = group
        if attention is None:
            from .attention import sparse_attention
            from .n8_v6 import N8V6Core

            self.core = N8V6Core(config)

            def attention(q, k, v):
                return sparse_attention(q, k, v, self.core)[0]

        self.attention = attention

    def __call__(self, q, k, v):
        qh, kh, vh = (seq_to_head(t, self.group) for t in (q, k, v))
        return head_to_seq(self.attention(qh, kh, vh), self.group)
