"""The adapter-facing SparsePR attention call and the Wan2.2 drop-in hook.

``sparse_attention`` mirrors ``_sparse_n8_attention_bhld``
(``src/sparsepr/adapters/wan22.py:1945-2182``): route, block-sparse
attention over the kept cluster pairs (stored straight back to the original
token order), then probe repair.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import kernels as K
from .n8_v6 import N8V6Config, N8V6Core

__all__ = ["sparse_attention", "route_phase", "attend_phase", "hunyuan_sparse_attention", "hunyuan_attend", "install_hunyuan_sparse_patch", "Wan22TI2VSparseConfig", "install_wan22_ti2v_sparse_patch", "make_n8_core",
           "kept_flops", "sparse_n8_attention_bhld"]


def sparse_attention(q, k, v, core: N8V6Core, *, total_key_tokens: int | None = None, attn_events=None,
                     return_base: bool = False, fused_repair: bool = True, **route_kw):
    """One SparsePR attention call on [B,H,N,D] Q/K/V.

    Returns ``(repaired [B,H,N,D] bf16, density float, info dict)`` like the
    reference's ``(repaired, density, timings)``.  With top-p budgets the
    density is a device scalar read once at the end (a 0-dim tensor while a
    CUDA graph is being captured).  ``info`` also holds the ``route`` and the
    ``repair_state``; ``attn_events`` (optional pair of ``torch.cuda.Event``)
    brackets the block-sparse attention launch on the current stream.

    The repair runs fused into the attention epilogue where the configuration
    allows it (``N8V6Core.fused_repair_supported``): a probe pre-pass computes
    the probe rows' exact and sparse outputs in one kernel, the state is
    fitted from them, and the attention kernel applies it (the rank-16
    correction on the tensor cores) and overwrites the probe rows before its
    store.  Otherwise, or with ``fused_repair=False``, the attention output is
    stored and ``N8V6Core.repair`` applies the repair.
    ``return_base`` also returns the unrepaired output as ``info["base"]``
    (an extra attention launch on the fused path; for tests).
    """
    route = route_phase(q, k, v, core, total_key_tokens=total_key_tokens, **route_kw)
    return attend_phase(q, k, v, core, route, attn_events=attn_events, return_base=return_base,
                        fused_repair=fused_repair)


def route_phase(q, k, v, core: N8V6Core, *, total_key_tokens: int | None = None, **route_kw):
    """The routing half of :func:`sparse_attention` (checks, the previous
    layer's status words, ``core.route``); returns the route."""
    if q.ndim != 4:
        raise RuntimeError(f"sparse_attention expects [B,H,N,D] tensors, got {tuple(q.shape)}.")
    batch, heads, tokens, dim = q.shape
    if batch != 1:
        raise RuntimeError("Wan2.2 N8 currently requires batch size one.")
    if q.is_cuda:
        K.raise_device_status(q.device)  # the previous layer's status words, if they have landed
    return core.route(q, k, v, total_key_tokens=tokens if total_key_tokens is None else total_key_tokens,
                      **route_kw)


def attend_phase(q, k, v, core: N8V6Core, route, *, attn_events=None, return_base: bool = False,
                 fused_repair: bool = True):
    """The attention half of :func:`sparse_attention` on a route from
    :func:`route_phase`: probe pre-pass, fit, block-sparse attention with the
    fused repair (or attention then ``core.repair``)."""
    batch, heads, tokens, dim = q.shape
    bh = batch * heads
    k_perm, v_perm = route.k_permuted.view(bh, -1, dim), route.v_permuted.view(bh, -1, dim)
    base = None
    if fused_repair and core.fused_repair_supported(route, dim):
        rows, weights = core.probe_rows(route)
        q3 = q.to(torch.bfloat16).contiguous().view(bh, tokens, dim)
        row_cluster = torch.gather(route.q_labels, 1, rows.long())
        dense, base_probe = K.probe_rows_attention(q3, k_perm, v_perm, route.k_offsets, route.extras["routed"], rows,
                                                   row_cluster)
        state, info = core.fit_repair(base_probe, dense, weights, tokens, route)
        if attn_events is not None:
            attn_events[0].record()
        repaired = K.block_sparse_attention(
            route.q_permuted, k_perm, v_perm, route.q_offsets, route.k_offsets, route.selected_ids,
            route.selected_counts, q_order=route.q_sorted_indices,
            repair=(state, core.config.repair_alpha, rows, dense))
        if attn_events is not None:
            attn_events[1].record()
        if return_base:
            base = K.block_sparse_attention(route.q_permuted, k_perm, v_perm, route.q_offsets, route.k_offsets,
                                            route.selected_ids, route.selected_counts, q_order=route.q_sorted_indices)
        repaired = repaired.view(batch, heads, tokens, dim)
        info["repair_fused"] = True
        info["probe_base"], info["probe_dense"] = base_probe, dense
    else:
        if attn_events is not None:
            attn_events[0].record()
        base = K.block_sparse_attention(route.q_permuted, k_perm, v_perm, route.q_offsets, route.k_offsets,
                                        route.selected_ids, route.selected_counts, q_order=route.q_sorted_indices)
        if attn_events is not None:
            attn_events[1].record()
        repaired, info = core.repair(base.view(batch, heads, tokens, dim), q, k, v, route)
        info["repair_fused"] = False
    K.collect_status(q.device)
    info["route"] = route
    info["base"] = base
    info["repair_state"] = core.repair_state_current
    density = info["effective_video_density"]
    if isinstance(density, torch.Tensor) and not torch.cuda.is_current_stream_capturing():
        density = float(density)  # top-p budgets: the one host read of the layer, as in the reference
    return repaired, density, info


def hunyuan_attend(query, key, value, core: N8V6Core, *, video_tokens: int, prompt_length: int):
    """Route and block-sparse attention of :func:`hunyuan_sparse_attention`
    before the repair: returns ``(attended [1,H,N,D] in token order, route,
    video queries)``.

    ``query/key/value`` [1,H,video+text,D]: video tokens first, then the text
    context (``prompt_length`` real prompt tokens, then padding).  Routing sees
    the video tokens (prompt keys always attended, the full K/V as permute
    source).  Two text clusters extend the map: every video query cluster
    also attends the prompt; the prompt rows attend every video key cluster
    and the prompt; padding rows attend only the padding.
    """
    if query.ndim != 4 or key.shape != query.shape or value.shape != query.shape:
        raise RuntimeError(f"Hunyuan SparsePR expects matching [B,H,N,D] tensors, got {tuple(query.shape)}, "
                           f"{tuple(key.shape)}, {tuple(value.shape)}.")
    batch, heads, tokens, dim = query.shape
    text = tokens - int(video_tokens)
    if batch != 1 or text < 0 or not 0 <= prompt_length <= text:
        raise RuntimeError(f"Hunyuan sequence mismatch: {tokens} tokens, video {video_tokens}, prompt {prompt_length}.")
    dev = query.device
    q_video = query[:, :, :video_tokens].contiguous()
    k_video = key[:, :, :video_tokens].contiguous()
    v_video = value[:, :, :video_tokens].contiguous()
    route = core.route(q_video, k_video, v_video, always_attended_keys=int(prompt_length),
                       total_key_tokens=int(video_tokens) + int(prompt_length), k_full_source=key,
                       v_full_source=value)
    if not route.permuted_includes_suffix:
        raise RuntimeError("SparsePR did not return the full Hunyuan K/V layout.")
    bh = batch * heads
    cq, ck = route.selected_ids.shape[1], route.selected_ids.shape[2]
    # Query order: video rows by cluster, text rows in place.
    suffix = torch.arange(video_tokens, tokens, device=dev, dtype=torch.int32).expand(bh, -1)
    q_order = torch.cat((route.q_sorted_indices.to(torch.int32), suffix), dim=1).contiguous()
    q_perm = K.permute_rows(query.to(torch.bfloat16).contiguous().view(bh, tokens, dim), q_order)
    # Cluster layout with the prompt and padding clusters appended to both sides.
    tail = torch.tensor([video_tokens + prompt_length, tokens], device=dev, dtype=torch.int32).expand(bh, -1)
    q_off = torch.cat((route.q_offsets.to(torch.int32), tail), dim=1).contiguous()
    k_off = torch.cat((route.k_offsets.to(torch.int32), tail), dim=1).contiguous()
    sel = torch.full((bh, cq + 2, ck + 2), -1, device=dev, dtype=torch.int32)
    sel[:, :cq, :ck] = route.selected_ids
    counts = torch.empty((bh, cq + 2), device=dev, dtype=torch.int32)
    sel[:, :cq].scatter_(2, route.selected_counts.long().unsqueeze(-1), ck)  # + prompt cluster (highest id)
    counts[:, :cq] = route.selected_counts + 1
    sel[:, cq, :ck + 1] = torch.arange(ck + 1, device=dev, dtype=torch.int32)  # prompt rows: all but padding
    counts[:, cq] = ck + 1
    sel[:, cq + 1, 0] = ck + 1  # padding rows: padding only
    counts[:, cq + 1] = 1
    out = K.block_sparse_attention(q_perm, route.k_permuted.view(bh, -1, dim), route.v_permuted.view(bh, -1, dim),
                                   q_off, k_off, sel, counts, q_order=q_order).view(batch, heads, tokens, dim)
    return out, route, q_video


def hunyuan_sparse_attention(query, key, value, core: N8V6Core, *, video_tokens: int, prompt_length: int):
    """SparsePR call of the HunyuanVideo processor (``hunyuanvideo.py:160-239``).

    ``query/key/value`` [1,H,video+text,D]: video tokens first, then the text
    context (``prompt_length`` real prompt tokens, then padding).  Routing sees
    the video tokens (prompt keys always attended, the full K/V as permute
    source).  Two text clusters extend the map: every video query cluster
    also attends the prompt; the prompt rows attend every video key cluster
    and the prompt; padding rows attend only the padding.  Video rows are
    repaired against K/V over video + prompt; text rows are returned as
    attended.  Returns ``[1,H,video+text,D]`` bf16.
    """
    out, route, q_video = hunyuan_attend(query, key, value, core, video_tokens=video_tokens,
                                         prompt_length=prompt_length)
    keep = int(video_tokens) + int(prompt_length)
    repaired, _info = core.repair(out[:, :, :video_tokens], q_video, key[:, :, :keep], value[:, :, :keep], route)
    return torch.cat((repaired, out[:, :, video_tokens:]), dim=2)


def install_hunyuan_sparse_patch(processor_cls, core_attr: str = "n8"):
    """Route ``processor_cls._sparse_attention`` (the reference's
    ``HunyuanVideoN8Processor``, ``hunyuanvideo.py:160-239``) through
    :func:`hunyuan_sparse_attention`.  The processor keeps its own core in
    ``core_attr``; it must be a ``sparsepr_b200.N8V6Core``.  Returns the
    previous method."""
    previous = getattr(processor_cls, "_sparse_attention", None)

    def _sparse_attention(self, query, key, value):
        return hunyuan_sparse_attention(query, key, value, getattr(self, core_attr),
                                        video_tokens=self.num_frame_patches * self.frame_size,
                                        prompt_length=self.prompt_length)

    processor_cls._sparse_attention = _sparse_attention
    return previous


def kept_flops(route, head_dim: int, probe_rows: int, tokens: int) -> torch.Tensor:
    """Kept FLOPs ``4*D*(selected_pairs + probe_pairs)`` as a device scalar
    (the reference FLOP audit, ``src/sparsepr/adapters/wan22.py:183-190, 2044-2065``)."""
    mask = route.video_dynamic_map
    sel_keys = (mask.long() * route.k_cluster_sizes.long().unsqueeze(1)).sum(-1)
    pairs = (sel_keys * route.q_cluster_sizes.long()).sum()
    probe_pairs = mask.shape[0] * probe_rows * tokens
    return 4 * head_dim * (pairs + probe_pairs)


@dataclass
class Wan22TI2VSparseConfig:
    """N8 fields of ``src/sparsepr/adapters/wan22.py:22-57`` used by the core."""

    num_q_centroids: int = 300
    num_k_centroids: int = 1000
    kmeans_iter_init: int = 50
    kmeans_iter_step: int = 2
    n8_target_density: float = 0.22
    n8_probe_rows: int = 64
    n8_repair_rank: int = 16
    n8_role_q_rank: int = 64
    n8_role_k_rank: int = 48
    n8_role_v_rank: int = 16
    n8_role_v_weight: float = 0.0
    n8_metric_sample_tokens: int = 2048
    n8_factor_power_iters: int = 2
    n8_factor_refresh_every: int = 1
    n8_role_kv_matmul_precision: str = "high"
    n8_selector_policy: str = "attention_mass"


_CONFIG = Wan22TI2VSparseConfig()


def make_n8_core(cfg: Wan22TI2VSparseConfig | None = None) -> N8V6Core:
    """``_make_n8_core`` (``wan22.py:1515-1548``) on this build."""
    c = cfg or _CONFIG
    return N8V6Core(N8V6Config(
        num_q_centroids=int(c.num_q_centroids), num_k_centroids=int(c.num_k_centroids),
        target_density=float(c.n8_target_density), role_q_rank=int(c.n8_role_q_rank),
        role_k_rank=int(c.n8_role_k_rank), role_v_rank=int(c.n8_role_v_rank),
        role_v_weight=float(c.n8_role_v_weight), metric_sample_tokens=int(c.n8_metric_sample_tokens),
        kmeans_iter_init=int(c.kmeans_iter_init), kmeans_iter_step=int(c.kmeans_iter_step),
        factor_power_iters=int(c.n8_factor_power_iters), factor_refresh_every=int(c.n8_factor_refresh_every),
        probe_rows=int(c.n8_probe_rows), repair_rank=int(c.n8_repair_rank),
        selector_policy=str(c.n8_selector_policy), role_kv_matmul_precision=str(c.n8_role_kv_matmul_precision),
    ))


def _core_for_cfg_branch(attn) -> N8V6Core:
    """Branch-local core per CFG pass (``wan22.py:1551-1566``)."""
    branch = int(getattr(attn, "_svg_cfg_branch", 0))
    cores = getattr(attn, "_n8_cores", None)
    if not isinstance(cores, dict):
        cores = {}
        attn._n8_cores = cores
    core = cores.get(branch)
    if core is None:
        core = make_n8_core()
        cores[branch] = core
    attn._n8_core = core
    return core


def sparse_n8_attention_bhld(attn, q_bhld, k_bhld, v_bhld, seq_lens=None):
    """Drop-in body of ``_sparse_n8_attention_bhld``: returns ``(repaired, density, timings)``."""
    del seq_lens
    core = _core_for_cfg_branch(attn)
    out, density, info = sparse_attention(q_bhld, k_bhld, v_bhld, core)
    for key in ("route", "base", "repair_state", "probe_base", "probe_dense"):
        info.pop(key, None)
    dtype = v_bhld.dtype if v_bhld.dtype in (torch.float16, torch.bfloat16) else torch.bfloat16
    return out.to(dtype), density, info


def install_wan22_ti2v_sparse_patch(config: Wan22TI2VSparseConfig | None = None, module=None,
                                    extension_module=None):
    """Install this build behind ``--attention sparsepr``.

    ``module`` is the reference adapter module (``sparsepr.adapters.wan22``);
    its ``_sparse_n8_attention_bhld`` is replaced by
    :func:`sparse_n8_attention_bhld` and its ``_make_n8_core`` by
    :func:`make_n8_core`, so the reference's Wan attention override routes
    every sparse call through sparsepr_b200.  ``extension_module`` (optional,
    ``sparsepr.kernels.n8_extension``) gets this build's
    ``wan_qkv_norm_rope_layout``, which the adapter's fused Q/K/V producer path
    (``SPARSEPR_N8_CUDA_EXT_WAN_QKV``) imports from there.  Returns the previous
    attention and core functions.
    """
    global _CONFIG
    if config is not None:
        _CONFIG = config
    if module is None:
        import importlib

        module = importlib.import_module("sparsepr.adapters.wan22")
    previous = (getattr(module, "_sparse_n8_attention_bhld", None), getattr(module, "_make_n8_core", None))
    module._sparse_n8_attention_bhld = sparse_n8_attention_bhld
    module._make_n8_core = make_n8_core
    if extension_module is not None:
        from .kernels import wan_qkv_norm_rope_layout

        extension_module.wan_qkv_norm_rope_layout = wan_qkv_norm_rope_layout
    return previous
