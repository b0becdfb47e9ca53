"""Route reuse across denoising steps and classifier-free-guidance branches.

Mirrors the Cosmos2.5 adapter's route cache (``src/sparsepr/adapters/
cosmos_predict2.py:138-145, 840-868, 1193-1400``): a sparse attention call
either refreshes its module's route (full ``N8V6Core.route``) or reuses the
cached one with the current step's Q/K/V.  A reuse skips clustering, the
role factors, the scorer and the selector: it permutes the current K, V and
Q by the cached key and query orders, runs the block-sparse attention over
the cached cluster-pair lists (already device-resident, so nothing is
re-planned) and repairs against the current Q/K/V with the cached probe
rows.

Steps before ``dense_first_steps`` run exact dense attention and leave the
cache untouched (``cosmos_predict2.py:1509-1520``); ``RouteCache.action``
reports them as ``"dense"``.  The action of a sparse call
(``cosmos_predict2.py:843-859``):

* no cached route                                   -> ``"refresh"``
* ``share_cfg_route`` and the route was last used in this same step
                                                    -> ``"cfg_reuse"``
* ``step - dense_first_steps`` negative or a multiple of
  ``route_refresh_every``                           -> ``"refresh"``
* otherwise                                         -> ``"temporal_reuse"``

The cache key is ``(module id, branch)``, with the branch folded to 0 when
``share_cfg_route`` (``cosmos_predict2.py:840-841``).  After each call the
cached route drops its step-sized tensors (permuted K/V/Q, role features)
and keeps the labels, orders, offsets, selection lists and probe rows
(``cosmos_predict2.py:862-868``).
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, field

import torch

from . import kernels as K
from .n8_v6 import N8V6Core, N8V6Route

__all__ = ["RouteReuseConfig", "RouteCache", "route_action"]


@dataclass
class RouteReuseConfig:
    """Route-reuse fields of ``Cosmos25N8Config`` (``cosmos_predict2.py:39, 53-54``)."""

    dense_first_steps: int = 2
    route_refresh_every: int = 4
    share_cfg_route: bool = True

    def validate(self) -> None:
        if self.dense_first_steps < 0:
            raise ValueError("dense_first_steps must lie in [0, total_steps].")
        if self.route_refresh_every <= 0:
            raise ValueError("route_refresh_every must be positive.")


@dataclass
class _Entry:
    """Cached route of one module (``_RouteCacheEntry``, ``cosmos_predict2.py:138-145``)."""

    origin_step: int
    last_step: int
    route: N8V6Route


def route_action(entry: _Entry | None, *, step: int, config: RouteReuseConfig) -> str:
    """``"refresh"``, ``"cfg_reuse"`` or ``"temporal_reuse"`` (``cosmos_predict2.py:843-859``)."""
    if entry is None:
        return "refresh"
    if config.share_cfg_route and entry.last_step == step:
        return "cfg_reuse"
    sparse_step = step - config.dense_first_steps
    if sparse_step < 0 or sparse_step % config.route_refresh_every == 0:
        return "refresh"
    return "temporal_reuse"


@dataclass
class RouteCache:
    """Per-module route cache in front of ``N8V6Core`` (one core per module).

    ``attention(q, k, v, core, module_id=, step=, branch=)`` returns
    ``(repaired [B,H,N,D] bf16, density, info)`` like
    :func:`sparsepr_b200.attention.sparse_attention`; ``info["route_action"]``
    says which action ran.  ``counts`` tallies the actions like the
    adapter's method counters."""

    config: RouteReuseConfig = field(default_factory=RouteReuseConfig)
    entries: dict = field(default_factory=dict)
    counts: dict = field(default_factory=lambda: {"route_refresh_calls": 0, "route_reuse_calls": 0,
                                                  "cfg_route_reuse_calls": 0, "temporal_route_reuse_calls": 0})

    def __post_init__(self):
        self.config.validate()

    def key(self, module_id, branch: int):
        return (module_id, 0 if self.config.share_cfg_route else int(branch))

    def action(self, module_id, *, step: int, branch: int = 0) -> str:
        if step < self.config.dense_first_steps:
            return "dense"
        return route_action(self.entries.get(self.key(module_id, branch)), step=step, config=self.config)

    def attention(self, q, k, v, core: N8V6Core, *, module_id, step: int, branch: int = 0,
                  attn_events=None, **route_kw):
        if q.ndim != 4 or k.shape != q.shape or v.shape != q.shape:
            raise RuntimeError(f"RouteCache expects matching [B,H,N,D] Q/K/V, got {tuple(q.shape)}, "
                               f"{tuple(k.shape)}, {tuple(v.shape)}.")
        batch, heads, tokens, dim = q.shape
        bh = batch * heads
        if step < self.config.dense_first_steps:
            # Forced-dense warm-up steps (cosmos_predict2.py:1509-1520): exact
            # attention, and the route cache is neither read nor written.
            dt = torch.bfloat16
            out = K.dense_attention_rows(q.to(dt).contiguous().view(bh, tokens, dim),
                                         k.to(dt).contiguous().view(bh, tokens, dim),
                                         v.to(dt).contiguous().view(bh, tokens, dim))
            self.counts["dense_calls"] = self.counts.get("dense_calls", 0) + 1
            return out.view(batch, heads, tokens, dim), 1.0, {"route_action": "dense"}
        key = self.key(module_id, branch)
        entry = self.entries.get(key)
        act = route_action(entry, step=step, config=self.config)
        if act == "refresh":
            route = core.route(q, k, v, total_key_tokens=tokens, **route_kw)
            entry = _Entry(origin_step=step, last_step=step, route=copy.copy(route))
            self.entries[key] = entry
            self.counts["route_refresh_calls"] += 1
        else:
            cached = entry.route
            if cached.permuted_includes_suffix:
                raise RuntimeError("Route reuse covers video-only routes (no text suffix in the K/V layout).")
            if cached.k_labels.shape != (bh, tokens):
                raise RuntimeError(f"Cached route covers {tuple(cached.k_labels.shape)} tokens; "
                                   f"this call has {(bh, tokens)}.")
            # The current step's K/V/Q in the cached cluster orders (cosmos_predict2.py:1310-1335).
            dt = torch.bfloat16
            kp = K.permute_rows(k.to(dt).contiguous().view(bh, tokens, dim), cached.k_sorted_indices)
            vp = K.permute_rows(v.to(dt).contiguous().view(bh, tokens, dim), cached.k_sorted_indices)
            qp = K.permute_rows(q.to(dt).contiguous().view(bh, tokens, dim), cached.q_sorted_indices)
            route = _with_tensors(cached, kp.view(batch, heads, tokens, dim), vp.view(batch, heads, tokens, dim), qp)
            entry.last_step = step
            self.counts["route_reuse_calls"] += 1
            self.counts["cfg_route_reuse_calls" if act == "cfg_reuse" else "temporal_route_reuse_calls"] += 1
        if attn_events is not None:
            attn_events[0].record()
        base = K.block_sparse_attention(
            route.q_permuted, route.k_permuted.view(bh, -1, dim), route.v_permuted.view(bh, -1, dim),
            route.q_offsets, route.k_offsets, route.selected_ids, route.selected_counts,
            q_order=route.q_sorted_indices)
        if attn_events is not None:
            attn_events[1].record()
        repaired, info = core.repair(base.view(batch, heads, tokens, dim), q, k, v, route)
        if route.probe_rows is not None and entry.route.probe_rows is None:
            entry.route.probe_rows, entry.route.probe_weights = route.probe_rows, route.probe_weights
        _compact(entry.route)
        info["route_action"] = act
        info["route"] = route
        info["base"] = base
        return repaired, float(info["effective_video_density"]), info


def _with_tensors(cached: N8V6Route, k_perm, v_perm, q_perm) -> N8V6Route:
    """A shallow copy of ``cached`` carrying this step's permuted tensors."""
    route = copy.copy(cached)
    route.k_permuted, route.v_permuted, route.q_permuted = k_perm, v_perm, q_perm
    return route


def _compact(route: N8V6Route) -> None:
    """Drop the step-sized tensors of a cached route (``cosmos_predict2.py:862-868``)."""
    route.k_permuted = route.v_permuted = route.q_permuted = None
    route.q_role_features = None
