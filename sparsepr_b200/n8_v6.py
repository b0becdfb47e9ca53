"""N8-V6 routing + repair core on the B200 kernels (drop-in for
``src/sparsepr/models/common/n8_v6.py``).

Same configuration fields, route/repair split and error messages as the
reference.  Small per-head linear algebra (role metrics, eigh factors, the
64x64 ridge fit) stays in PyTorch/cuSOLVER; every token-sized step runs in
the sparsepr_b200 CUDA library: Lloyd k-means, label sort, centroid means
fused with the K/V/Q permutes, selector scores, budgeted selection, block
sparse attention, dense probe rows and the repair apply.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import kernels as K
from .synthetic import random_init_indices

__all__ = ["N8V6Config", "N8V6Route", "N8V6Core"]


@dataclass(frozen=True)
class N8V6Config:
    """Immutable N8-V6 method configuration (fields of ``n8_v6.py:233-280``).

    Fields that select reference-only backends (Triton block sizes, warps,
    ``kmeans_backend``, ``compile_role_kv_projection``) are accepted for
    drop-in compatibility and have no effect here.  Added fields:
    ``kmeans_tol`` (the reference's implicit ``batch_kmeans_Euclid`` default
    1e-4), ``kmeans_init_seed`` (seed of the cold-start random-sample init)
    and ``kmeans_precision`` ("tf32" like the reference's Triton ``tl.dot``,
    or "fp32" for 3xTF32 distances that match an fp32 reference bit for bit
    away from near ties).
    """

    num_q_centroids: int = 300
    num_k_centroids: int = 1000
    target_density: float = 0.22
    role_q_rank: int = 64
    role_k_rank: int = 48
    role_v_rank: int = 16
    role_v_weight: float = 0.0
    metric_sample_tokens: int = 2048
    kmeans_iter_init: int = 25
    kmeans_iter_step: int = 2
    kmeans_backend: str = "flash"
    factor_power_iters: int = 2
    factor_orthogonalization: str = "each_cholesky_qr2"
    factor_ritz_mode: str = "rayleigh_cholesky"
    factor_rayleigh_ridge: float = 1e-4
    factor_cholesky_qr_ridge: float = 1e-5
    factor_refresh_every: int = 1
    probe_rows: int = 64
    repair_rank: int = 16
    repair_ridge: float = 0.1
    repair_alpha: float = 1.0
    repair_norm_cap: float = 0.0
    repair_features: str = "output"
    repair_basis_source: str = "raw_residual"
    probe_selection_policy: str = "role_equal_centroid"
    selector_block_q: int = 32
    selector_block_n: int = 16
    selector_num_warps: int = 2
    selector_policy: str = "svg_ear_value"
    selector_budget_mode: str = "fixed_density"
    svg_ear_top_p: float = 0.85
    adaptive_budget_min_density: float = 0.0
    adaptive_budget_max_density: float = 1.0
    grouped_svg_ear_router: bool = False
    role_projection_block_m: int = 32
    role_projection_num_warps: int = 2
    repair_block_n: int = 16
    repair_num_warps: int = 2
    repair_num_stages: int = 1
    repair_input_precision: str = "tf32"
    compile_role_kv_projection: bool = True
    role_kv_matmul_precision: str = "high"
    profile_breakdown: bool = False
    kmeans_tol: float = 1e-4
    kmeans_init_seed: int = 0
    kmeans_precision: str = "tf32"

    def validate(self, head_dim: int | None = None) -> None:
        """Same checks and messages as ``n8_v6.py:281-348``."""
        if not 0.0 < self.target_density <= 1.0:
            raise ValueError(f"target_density must be in (0,1], got {self.target_density}.")
        if self.probe_rows <= 0 or self.repair_rank <= 0:
            raise ValueError("N8 probe_rows and repair_rank must be positive.")
        if self.factor_refresh_every <= 0:
            raise ValueError("factor_refresh_every must be positive.")
        if self.role_kv_matmul_precision not in {"highest", "high", "medium"}:
            raise ValueError(
                "role_kv_matmul_precision must be highest, high, or medium; got "
                f"{self.role_kv_matmul_precision!r}."
            )
        if self.probe_rows > self.num_q_centroids:
            raise ValueError("Vectorized role-equal probes require M <= Q clusters.")
        if self.role_v_weight < 0.0:
            raise ValueError("role_v_weight must be non-negative.")
        if self.repair_norm_cap < 0.0:
            raise ValueError("repair_norm_cap must be non-negative.")
        if self.repair_features not in {"output", "output_role"}:
            raise ValueError(f"repair_features must be output or output_role; got {self.repair_features!r}.")
        if self.repair_basis_source not in {"raw_residual", "fitted_residual"}:
            raise ValueError(
                f"repair_basis_source must be raw_residual or fitted_residual; got {self.repair_basis_source!r}."
            )
        if self.selector_policy not in {"svg_ear_value", "attention_mass"}:
            raise ValueError(
                f"selector_policy must be svg_ear_value or attention_mass; got {self.selector_policy!r}."
            )
        if self.selector_budget_mode not in {"fixed_density", "svg_ear_top_p"}:
            raise ValueError(
                f"selector_budget_mode must be fixed_density or svg_ear_top_p; got {self.selector_budget_mode!r}."
            )
        if not 0.0 < self.svg_ear_top_p <= 1.0:
            raise ValueError(f"svg_ear_top_p must be in (0,1], got {self.svg_ear_top_p}.")
        if not (0.0 <= self.adaptive_budget_min_density <= self.adaptive_budget_max_density <= 1.0):
            raise ValueError(
                "Adaptive budget densities must satisfy 0 <= minimum <= maximum <= 1; got "
                f"minimum={self.adaptive_budget_min_density}, maximum={self.adaptive_budget_max_density}."
            )
        if self.kmeans_precision not in {"tf32", "fp32"}:
            raise ValueError(f"kmeans_precision must be tf32 or fp32; got {self.kmeans_precision!r}.")
        if self.probe_selection_policy not in {"role_equal_centroid", "first_token_largest_groups"}:
            raise ValueError(
                "probe_selection_policy must be role_equal_centroid or first_token_largest_groups; got "
                f"{self.probe_selection_policy!r}."
            )
        if head_dim is not None and max(self.role_q_rank, self.role_k_rank, self.role_v_rank) > head_dim:
            raise ValueError(f"N8 role rank exceeds head dimension {head_dim}.")


@dataclass
class N8V6Route:
    """Routing result (fields of ``n8_v6.py:351-369``) plus the device schedule
    the B200 attention kernel consumes (offsets, orders, compacted selection).

    Labels and sizes are int32 (the reference uses int64).  ``q_kmeans_iters``
    / ``k_kmeans_iters`` hold the requested iteration count; the executed
    count (smaller when ``kmeans_tol`` stopped a run) stays on the device in
    ``extras['q_iters_done']`` / ``extras['k_iters_done']`` so routing never
    synchronises with the host.
    """

    q_labels: torch.Tensor
    k_labels: torch.Tensor
    q_cluster_sizes: torch.Tensor
    k_cluster_sizes: torch.Tensor
    video_dynamic_map: torch.Tensor
    q_role_features: torch.Tensor
    k_permuted: torch.Tensor
    v_permuted: torch.Tensor
    k_sorted_indices: torch.Tensor
    base_video_density: float
    q_kmeans_iters: int
    k_kmeans_iters: int
    permuted_includes_suffix: bool = False
    probe_rows: torch.Tensor | None = None
    probe_weights: torch.Tensor | None = None
    q_sorted_indices: torch.Tensor | None = None
    q_permuted: torch.Tensor | None = None
    q_offsets: torch.Tensor | None = None
    k_offsets: torch.Tensor | None = None
    selected_ids: torch.Tensor | None = None
    selected_counts: torch.Tensor | None = None
    scores: torch.Tensor | None = None
    budgets: torch.Tensor | None = None
    extras: dict = field(default_factory=dict)


# ----------------------------------------------------------------------------
# Small per-head linear algebra (PyTorch / cuSOLVER on the device)
# ----------------------------------------------------------------------------

_DEVICE_CONST: dict[tuple, torch.Tensor] = {}


def _device_const(key: tuple, make) -> torch.Tensor:
    """Small constant index tensors built once on the host and cached per device,
    so a route call never issues a blocking host-to-device copy."""
    t = _DEVICE_CONST.get(key)
    if t is None:
        t = make()
        _DEVICE_CONST[key] = t
    return t


def _sample_positions(tokens: int, sample_tokens: int, device) -> torch.Tensor | None:
    """Evenly spaced token positions (``operator_kmeans.py:52-59``)."""
    if sample_tokens <= 0 or sample_tokens >= tokens:
        return None
    return _device_const(
        ("sample", tokens, sample_tokens, str(device)),
        lambda: torch.linspace(0, tokens - 1, steps=sample_tokens).round().long().unique(sorted=True).to(device))


def _init_indices(bh: int, tokens: int, k: int, seed: int, device) -> torch.Tensor:
    return _device_const(("init", bh, tokens, k, seed, str(device)),
                         lambda: random_init_indices(bh, tokens, k, seed).to(device))


def _projection_kernel_fits(dim: int, rank: int) -> bool:
    """Shapes served by the tensor-core role projection (``spr_role_projection``);
    other shapes project with torch matmuls on the GPU."""
    return dim == 128 and rank in (16, 32, 48, 64)


def key_metric_from_queries(q: torch.Tensor, sample_tokens: int) -> torch.Tensor:
    """Uncentered fp32 covariance of sampled queries (``operator_kmeans.py:491-493``)."""
    pos = _sample_positions(q.shape[1], sample_tokens, q.device)
    s = (q if pos is None else q[:, pos]).float()
    return torch.bmm(s.transpose(1, 2), s) / max(int(s.shape[1]), 1)


def query_metric_from_key_centroids(centroids: torch.Tensor, sizes: torch.Tensor) -> torch.Tensor:
    """Centered metric of the non-empty key centroids (``operator_kmeans.py:514-529``)."""
    valid = (sizes > 0).float()
    count = valid.sum(dim=1).clamp_min(1.0)
    mean = (centroids.float() * valid.unsqueeze(-1)).sum(dim=1) / count.unsqueeze(-1)
    cen = (centroids.float() - mean.unsqueeze(1)) * valid.unsqueeze(-1)
    return torch.bmm(cen.transpose(1, 2), cen) / count.view(-1, 1, 1) / float(centroids.shape[-1])


def metric_factor(metric: torch.Tensor, rank: int) -> torch.Tensor:
    """Top-``rank`` eigenvectors scaled by sqrt(eigenvalue/mean) (``operator_kmeans.py:94-151``)."""
    if metric.ndim != 3 or metric.shape[1] != metric.shape[2]:
        raise RuntimeError(f"Expected batched square metrics, got {tuple(metric.shape)}.")
    if rank <= 0 or rank > metric.shape[-1]:
        raise RuntimeError(f"rank must be in [1, {metric.shape[-1]}], got {rank}.")
    evals, evecs = K.sym_eig(metric.float(), top=rank)  # symmetrised inside the kernel
    evals = evals[:, -rank:].clamp_min(0.0)
    evecs = evecs[:, :, -rank:]
    norm = evals.mean(dim=1, keepdim=True).clamp_min(1e-12)
    return evecs * torch.sqrt(evals / norm).unsqueeze(1)


def warm_subspace_metric_factor(metric: torch.Tensor, previous: torch.Tensor, rank: int, *, power_iters: int = 2,
                                orthogonalization: str = "each_cholesky_qr2", ritz_mode: str = "rayleigh_cholesky",
                                rayleigh_ridge: float = 1e-4, cholesky_qr_ridge: float = 1e-5):
    """Warm top-``rank`` metric factor by subspace iteration from the previous
    basis (``operator_kmeans.py:221-477``): ``power_iters`` applications of the
    metric, each followed by Cholesky-QR (and a second, corrective one at the
    end for ``each_cholesky_qr2``), then the Ritz step: ``B chol(B^T M B)/sqrt(mean
    diag)`` (``rayleigh_cholesky``) or the reduced eigendecomposition (``full``).
    Returns ``(factor, basis, recovered)``; ``recovered`` marks heads whose
    Cholesky failed or whose result is not finite."""
    if metric.ndim != 3 or metric.shape[1] != metric.shape[2]:
        raise RuntimeError(f"Expected batched square metrics, got {tuple(metric.shape)}.")
    expected = (metric.shape[0], metric.shape[1], rank)
    if tuple(previous.shape) != expected:
        raise RuntimeError(f"Previous factor shape mismatch: got {tuple(previous.shape)}, expected {expected}.")
    if power_iters < 1:
        raise RuntimeError(f"power_iters must be positive, got {power_iters}.")
    if orthogonalization not in {"each_cholesky_qr", "each_cholesky_qr2"} or ritz_mode not in {"rayleigh_cholesky",
                                                                                            "full"}:
        raise NotImplementedError(
            "sparsepr_b200 implements warm factors with each_cholesky_qr[2] orthogonalization and "
            f"rayleigh_cholesky / full Ritz steps; got {orthogonalization!r}, {ritz_mode!r}.")
    m = metric.float()
    basis = previous.float()
    basis = basis / torch.linalg.vector_norm(basis, dim=1, keepdim=True).clamp_min(1e-12)
    recovered = torch.zeros(m.shape[0], dtype=torch.bool, device=m.device)
    for it in range(power_iters):
        basis, failed = K.cholesky_qr(torch.bmm(m, basis), cholesky_qr_ridge)
        recovered |= failed
        if orthogonalization == "each_cholesky_qr2" and it == power_iters - 1:
            basis, failed = K.cholesky_qr(basis, max(float(cholesky_qr_ridge), 1e-5))
            recovered |= failed
    rayleigh = torch.bmm(basis.transpose(1, 2), torch.bmm(m, basis))
    rayleigh = 0.5 * (rayleigh + rayleigh.transpose(1, 2))
    if ritz_mode == "rayleigh_cholesky":
        normalizer = rayleigh.diagonal(dim1=1, dim2=2).mean(dim=1).clamp_min(1e-12)
        chol, failed = K.ridge_cholesky(rayleigh, normalizer, rayleigh_ridge, 1e-2)
        recovered |= failed
        factor = torch.bmm(basis, chol) / torch.sqrt(normalizer)[:, None, None]
    else:
        evals, rot = K.sym_eig(rayleigh)
        evals = evals.clamp_min(0.0)
        normalizer = evals.mean(dim=1, keepdim=True).clamp_min(1e-12)
        factor = torch.bmm(basis, rot) * torch.sqrt(evals / normalizer).unsqueeze(1)
    recovered |= ~torch.isfinite(factor).all(dim=(1, 2)) | ~torch.isfinite(basis).all(dim=(1, 2))
    return factor, basis, recovered


class _MatmulPrecision:
    def __init__(self, precision: str):
        self.precision = precision

    def __enter__(self):
        self.prev = torch.get_float32_matmul_precision()
        torch.set_float32_matmul_precision(self.precision)

    def __exit__(self, *exc):
        torch.set_float32_matmul_precision(self.prev)


def select_role_equal_probes(role_features, role_labels, num_clusters: int, rows: int, *, order=None,
                             offsets=None):
    """One representative per largest role group (``residual_repair.py:118-208``).

    With the k-means sort (``order`` [BH,N] and ``offsets`` [BH,K+1], int32) the
    token pass (cluster means of the role features and the nearest token) is one
    kernel, ``spr_probe_representatives``, summing in a fixed order."""
    if role_features.ndim != 3 or role_labels.shape != role_features.shape[:2]:
        raise RuntimeError(
            "Role probe selection expects features [BH,N,R] and labels [BH,N], got "
            f"features={tuple(role_features.shape)}, labels={tuple(role_labels.shape)}."
        )
    bh, n, r = role_features.shape
    count = min(max(1, int(rows)), n)
    if count > int(num_clusters):
        raise RuntimeError(
            f"Vectorized role probes currently require rows <= num_clusters; got rows={count}, clusters={num_clusters}."
        )
    dev = role_features.device
    labels = role_labels.long()
    tok = torch.arange(n, device=dev).view(1, -1).expand(bh, -1)
    if order is not None and offsets is not None and r <= 64 and offsets.shape[-1] == num_clusters + 1:
        sizes = (offsets[:, 1:] - offsets[:, :-1]).long()
        best_idx = K.probe_representatives(role_features, order.to(torch.int32).contiguous(),
                                           offsets.to(torch.int32).contiguous()).long()
    else:
        feats = role_features.float()
        sizes = torch.zeros((bh, num_clusters), device=dev, dtype=torch.long)
        sizes.scatter_add_(1, labels, torch.ones_like(labels))
        sums = torch.zeros((bh, num_clusters, r), device=dev, dtype=torch.float32)
        sums.scatter_add_(1, labels.unsqueeze(2).expand(-1, -1, r), feats)
        centers = sums / sizes.clamp_min(1).unsqueeze(2)
        dist = (feats - torch.gather(centers, 1, labels.unsqueeze(2).expand(-1, -1, r))).square().sum(2)
        best = torch.full((bh, num_clusters), float("inf"), device=dev)
        best.scatter_reduce_(1, labels, dist, reduce="amin", include_self=True)
        cand = torch.where(dist == torch.gather(best, 1, labels), tok, torch.full_like(tok, n))
        best_idx = torch.full((bh, num_clusters), n, device=dev, dtype=torch.long)
        best_idx.scatter_reduce_(1, labels, cand, reduce="amin", include_self=True)
    order = torch.argsort(sizes, dim=1, descending=True, stable=True)
    sel = torch.gather(best_idx, 1, order)[:, :count]
    sel = torch.where(sel < n, sel, tok[:, :count])
    sel_labels = torch.gather(labels, 1, sel)
    sampled = torch.zeros_like(sizes)
    sampled.scatter_add_(1, sel_labels, torch.ones_like(sel_labels))
    gw = sizes.float() / sampled.clamp_min(1).float()
    w = torch.gather(gw, 1, sel_labels)
    return sel, w / w.mean(dim=1, keepdim=True).clamp_min(1e-20)


def select_first_token_largest_groups(role_features, role_labels, num_clusters: int, rows: int):
    """First token of each of the largest role groups (``residual_repair.py:211-260``)."""
    bh, n, _ = role_features.shape
    count = min(max(1, int(rows)), n)
    if count > int(num_clusters):
        raise RuntimeError(f"First-token role probes require rows <= num_clusters; got rows={count}, clusters={num_clusters}.")
    dev = role_labels.device
    labels = role_labels.long()
    sizes = torch.zeros((bh, num_clusters), device=dev, dtype=torch.long)
    sizes.scatter_add_(1, labels, torch.ones_like(labels))
    tok = torch.arange(n, device=dev).view(1, -1).expand(bh, -1)
    first = torch.full((bh, num_clusters), n, device=dev, dtype=torch.long)
    first.scatter_reduce_(1, labels, tok, reduce="amin", include_self=True)
    order = torch.argsort(sizes, dim=1, descending=True, stable=True)
    sel = torch.gather(first, 1, order)[:, :count]
    sel = torch.where(sel < n, sel, tok[:, :count])
    ssz = torch.gather(sizes, 1, torch.gather(labels, 1, sel)).float()
    return sel, ssz / ssz.mean(dim=1, keepdim=True).clamp_min(1e-20)


def _clamp_density(d):
    """min(1, d) for a float or a 0-dim device tensor (top-p budgets keep the
    density on the device)."""
    return d.clamp(max=1.0) if isinstance(d, torch.Tensor) else min(1.0, d)


def fit_reduced_rank_residual(x_fit, y_fit, weights, rank: int, ridge: float):
    """Weighted ridge RRR, dual Cholesky, raw-residual basis (``residual_repair.py:317-465``).

    Unlike the reference no device assert is raised on a failed Cholesky
    (``residual_repair.py:399-402`` traps the CUDA context): the non-finite
    state is replaced per head by ``recover_nonfinite_rrr_state``.
    """
    x = x_fit.float()
    y = y_fit.float()
    if rank <= 0 or rank > y.shape[2] or rank > x.shape[1]:
        raise RuntimeError(f"Invalid RRR rank={rank} for X={tuple(x.shape)}, Y={tuple(y.shape)}.")
    w = weights.float().unsqueeze(2)
    w_sum = w.sum(dim=1, keepdim=True).clamp_min(1e-20)
    x_mean = (w * x).sum(dim=1, keepdim=True) / w_sum
    x_var = (w * (x - x_mean).square()).sum(dim=1, keepdim=True) / w_sum
    x_scale = x_var.sqrt().clamp_min(1e-5)
    y_mean = (w * y).sum(dim=1, keepdim=True) / w_sum
    sw = w.sqrt()
    xw = (x - x_mean) / x_scale * sw
    yw = (y - y_mean) * sw
    m = x.shape[1]
    if m >= x.shape[2]:
        raise RuntimeError("The dual RRR fit needs fewer probe rows than features.")
    gram = torch.bmm(xw, xw.transpose(1, 2))
    gram.diagonal(dim1=1, dim2=2).add_(float(ridge))
    dual = K.chol_solve(gram, yw)
    evals, evecs = K.sym_eig(torch.bmm(yw, yw.transpose(1, 2)), top=rank)
    evecs = evecs[:, :, -rank:]
    scales = evals[:, -rank:].clamp_min(1e-20).rsqrt().unsqueeze(1)
    basis = (torch.bmm(yw.transpose(1, 2), evecs) * scales).contiguous()
    left = torch.bmm(xw.transpose(1, 2), torch.bmm(dual, basis)).contiguous()
    return x_mean, x_scale, y_mean, left, basis


def recover_nonfinite_rrr_state(state, previous):
    """Per-head recovery of a non-finite fit (``residual_repair.py:509-587``)."""
    bh = int(state[0].shape[0])
    recovered = torch.zeros(bh, device=state[0].device, dtype=torch.bool)
    for t in state:
        recovered |= ~torch.isfinite(t).reshape(bh, -1).all(dim=1)
    if previous is None:
        fallback = (torch.zeros_like(state[0]), torch.ones_like(state[1]), torch.zeros_like(state[2]),
                    torch.zeros_like(state[3]), torch.zeros_like(state[4]))
        policy = "zero_repair_without_previous_state"
    else:
        if len(previous) != len(state) or any(o.shape != n.shape for o, n in zip(previous, state)):
            raise RuntimeError("Previous RRR state does not match the current fit.")
        fallback = previous
        policy = "reuse_previous_finite_repair_state"
    sel = tuple(torch.where(recovered.reshape(bh, *((1,) * (c.ndim - 1))), o, c) for c, o in zip(state, fallback))
    return sel, recovered, policy


def _svg_top_p_key_budgets(q_centroids, k_centroids, k_sizes, top_p: float) -> torch.Tensor:
    """SVG2-style cumulative-mass key budgets per query cluster (``n8_v6.py:181-230``)."""
    if not 0.0 < float(top_p) <= 1.0:
        raise ValueError(f"svg_ear_top_p must be in (0,1], got {top_p}.")
    dim = int(q_centroids.shape[2])
    logits = torch.bmm(q_centroids.float(), k_centroids.float().transpose(1, 2)) / math.sqrt(dim)
    weights = k_sizes.float().unsqueeze(1)
    logits = logits - logits.amax(dim=2, keepdim=True)
    wexp = logits.exp() * weights
    prob = wexp / wexp.sum(dim=2, keepdim=True).clamp_min(1e-12)
    sp, order = torch.sort(prob, dim=2, descending=True, stable=True)
    keep = sp.cumsum(dim=2) <= float(top_p)
    keep = torch.nn.functional.pad(keep[:, :, :-1], (1, 0), value=True)
    ss = torch.gather(k_sizes.long().unsqueeze(1).expand(-1, q_centroids.shape[1], -1), 2, order)
    return (ss * keep.long()).sum(dim=2)


# ----------------------------------------------------------------------------
# The stateful core
# ----------------------------------------------------------------------------

class N8V6Core:
    """Stateful per-attention-layer N8-V6 core (``n8_v6.py:372-1444``).

    Cross-step state (previous original-space centroids and repair state) is
    kept like the reference: a second call warm-starts both k-means runs from
    the projected previous centroids with ``kmeans_iter_step`` iterations.
    Role factors are exact (eigh) on the first call and updated by the
    reference's warm subspace iteration (``operator_kmeans.py:221-477``) on
    later refreshes.
    """

    def __init__(self, config: N8V6Config, init_indices: tuple[torch.Tensor, torch.Tensor] | None = None):
        """``init_indices`` (extension): device tensors ``(k_idx [BH,Ck], q_idx [BH,Cq])``
        of cold-start centroid rows, used instead of ``random_init_indices``
        (a caller running a subset of the heads passes its rows of the full
        draw, so its results match a call over all heads)."""
        config.validate()
        self.config = config
        self.init_indices = init_indices
        self.q_centroids: torch.Tensor | None = None
        self.k_centroids: torch.Tensor | None = None
        self.v_centroids: torch.Tensor | None = None
        self.q_factor_current: torch.Tensor | None = None
        self.k_factor_current: torch.Tensor | None = None
        # Warm subspace bases the next factor update starts from (n8_v6.py:381-383).
        self.q_factor_state: torch.Tensor | None = None
        self.k_factor_state: torch.Tensor | None = None
        self.q_factor_recovery_mask: torch.Tensor | None = None
        self.k_factor_recovery_mask: torch.Tensor | None = None
        self.repair_state_current = None
        self.repair_recovery_mask: torch.Tensor | None = None
        self.route_call_index = 0
        self.last_route_profile: dict = {}
        self.last_repair_profile: dict = {}
        self.diagnostic_callback = None

    def _updated_factor(self, metric, previous, current, rank):
        """Exact factor on the first update, warm subspace iteration afterwards;
        a head whose warm solve fails keeps its previous factor and basis
        (``n8_v6.py:478-519``).  Returns ``(factor, state, recovered)``."""
        cfg = self.config
        if previous is None:
            factor = metric_factor(metric, rank)
            return factor, factor, torch.zeros(metric.shape[0], dtype=torch.bool, device=metric.device)
        if current is None:
            raise RuntimeError("Warm role-factor state is missing its current factor.")
        factor, state, recovered = warm_subspace_metric_factor(
            metric, previous, rank, power_iters=cfg.factor_power_iters,
            orthogonalization=cfg.factor_orthogonalization, ritz_mode=cfg.factor_ritz_mode,
            rayleigh_ridge=cfg.factor_rayleigh_ridge, cholesky_qr_ridge=cfg.factor_cholesky_qr_ridge)
        sel = recovered[:, None, None]
        return torch.where(sel, current.float(), factor), torch.where(sel, previous.float(), state), recovered

    @property
    def initialized(self) -> bool:
        return self.q_centroids is not None

    def reset(self) -> None:
        self.__init__(self.config, self.init_indices)

    # -- route ---------------------------------------------------------------
    def route(self, q_video, k_video, v_video, *, gqa_group_size: int = 1, always_attended_keys: int = 0,
              total_key_tokens: int | None = None, k_full_source=None, v_full_source=None,
              k_init_features=None, q_init_features=None) -> N8V6Route:
        """Build the cluster-pair route (``n8_v6.py:521-1172``, attention-mass selector).

        ``k_init_features``/``q_init_features`` (extension) override the
        initial centroids in role-feature space; by default a cold call uses
        the rows at ``random_init_indices(seed)`` and a warm call the
        projected previous centroids.
        """
        if q_video.shape != k_video.shape or q_video.shape != v_video.shape or q_video.ndim != 4:
            raise RuntimeError(
                "N8-V6 expects matching [B,H,N,D] video Q/K/V; got "
                f"Q={tuple(q_video.shape)}, K={tuple(k_video.shape)}, V={tuple(v_video.shape)}."
            )
        if not q_video.is_cuda:
            raise RuntimeError("sparsepr_b200 N8-V6 routing runs on CUDA tensors only (no CPU path).")
        batch, heads, tokens, dim = q_video.shape
        cfg = self.config
        cfg.validate(dim)
        group = int(gqa_group_size)
        if group <= 0 or heads % group:
            raise ValueError(f"gqa_group_size must divide the query-head count; got H={heads}, G={group}.")
        if cfg.role_v_weight != 0.0:
            raise NotImplementedError("role_v_weight > 0 is not implemented in sparsepr_b200.")
        bh = batch * heads
        kv_heads = heads // group
        bkv = batch * kv_heads
        dev = q_video.device
        dt = torch.bfloat16
        q = q_video.to(dt).contiguous().view(bh, tokens, dim)
        k_all = k_video.to(dt).contiguous()
        v_all = v_video.to(dt).contiguous()
        if group > 1:
            # GQA (n8_v6.py:549-567): K/V are clustered once per native KV head
            # (the first query head of each group); the key metric pools the
            # queries of the whole group, sampling group x as many tokens.
            k = k_all[:, ::group].contiguous().view(bkv, tokens, dim)
            v = v_all[:, ::group].contiguous().view(bkv, tokens, dim)
            k_metric_q = q.view(bkv, group * tokens, dim)
        else:
            k = k_all.view(bh, tokens, dim)
            v = v_all.view(bh, tokens, dim)
            k_metric_q = q
        k_all, v_all = k_all.view(bh, tokens, dim), v_all.view(bh, tokens, dim)
        warm = self.initialized
        iters = cfg.kmeans_iter_step if warm else cfg.kmeans_iter_init

        # Key role factor and features: K F_k / rms (n8_v6.py:612-681).  Factors
        # are refreshed on the first call and every factor_refresh_every calls.
        refresh = (self.q_factor_current is None or self.k_factor_current is None
                   or self.route_call_index % cfg.factor_refresh_every == 0)
        if refresh:
            k_factor, self.k_factor_state, self.k_factor_recovery_mask = self._updated_factor(
                key_metric_from_queries(k_metric_q, cfg.metric_sample_tokens * group), self.k_factor_state,
                self.k_factor_current, cfg.role_k_rank)
        else:
            k_factor = self.k_factor_current
        self.k_factor_current = k_factor
        with _MatmulPrecision(cfg.role_kv_matmul_precision):
            if _projection_kernel_fits(dim, k_factor.shape[-1]):
                k_feat, k_scale = K.role_projection(k, k_factor, "global")
            else:
                k_feat = torch.bmm(k.float(), k_factor)
                k_scale = k_feat.square().mean(dim=(1, 2), keepdim=True).sqrt().clamp_min(1e-8)
                k_feat = (k_feat / k_scale).contiguous()
            if k_init_features is None and warm:
                k_init_features = torch.bmm(self.k_centroids, k_factor) / k_scale
        if k_init_features is None:
            idx = (self.init_indices[0] if self.init_indices is not None
                   else _init_indices(bkv, tokens, cfg.num_k_centroids, cfg.kmeans_init_seed, dev))
            k_init_features = torch.gather(k_feat, 1, idx.unsqueeze(-1).expand(-1, -1, k_feat.shape[-1]))
        k_labels, _kc, k_sizes, k_off, k_order, k_it = K.kmeans_lloyd(k_feat, k_init_features, iters, cfg.kmeans_tol,
                                                                     precision=cfg.kmeans_precision)

        # Original-space K/V centroids fused with the K/V permute (n8_v6.py:734-741, 905-934).
        use_full = k_full_source is not None or v_full_source is not None
        fused_perm = not use_full and group == 1
        k_cent, k_perm = K.centroid_means(k, k_order, k_off, cfg.num_k_centroids, self.k_centroids, permute=fused_perm)
        v_cent, v_perm = K.centroid_means(v, k_order, k_off, cfg.num_k_centroids, self.v_centroids, permute=fused_perm)
        k_sizes_native = k_sizes
        if group > 1:
            # Native-head clustering copied to every query head of its group
            # (n8_v6.py:808-834); each query head then permutes its own K/V
            # rows with the group's order (n8_v6.py:905-934).
            def per_query_head(t):
                return t.view(batch, kv_heads, *t.shape[1:]).repeat_interleave(group, dim=1).reshape(
                    bh, *t.shape[1:]).contiguous()

            k_labels, k_sizes, k_off, k_order = (per_query_head(t) for t in (k_labels, k_sizes, k_off, k_order))
            if not use_full:
                k_perm = K.permute_rows(k_all, k_order)
                v_perm = K.permute_rows(v_all, k_order)
        if use_full:
            if k_full_source is None or v_full_source is None:
                raise ValueError("k_full_source and v_full_source must be provided together.")
            if k_full_source.shape != v_full_source.shape or k_full_source.ndim != 4:
                raise ValueError("Full K/V sources must have matching [B,H,N,D] shapes.")
            if tuple(k_full_source.shape[:2]) != (batch, heads) or k_full_source.shape[-1] != dim:
                raise ValueError("Full K/V sources do not match the video tensor head layout.")
            total_layout = int(k_full_source.shape[2])
            if total_layout < tokens:
                raise ValueError("Full K/V source is shorter than the video prefix.")
            suffix = torch.arange(tokens, total_layout, device=dev, dtype=torch.int32).expand(bh, -1)
            full_order = torch.cat((k_order, suffix), dim=1).contiguous()
            k_perm = K.permute_rows(k_full_source.to(dt).contiguous().view(bh, total_layout, dim), full_order)
            v_perm = K.permute_rows(v_full_source.to(dt).contiguous().view(bh, total_layout, dim), full_order)
        self.k_centroids, self.v_centroids = k_cent, v_cent

        # Query role factor from the key-centroid metric, row-RMS features (n8_v6.py:744-806).
        if refresh:
            q_factor, self.q_factor_state, self.q_factor_recovery_mask = self._updated_factor(
                query_metric_from_key_centroids(k_cent, k_sizes_native), self.q_factor_state, self.q_factor_current,
                cfg.role_q_rank)
        else:
            q_factor = self.q_factor_current
        self.q_factor_current = q_factor
        if group > 1:  # n8_v6.py:762-769: the group's Q factor on each query head
            q_factor = q_factor.view(batch, kv_heads, dim, -1).repeat_interleave(group, dim=1).reshape(bh, dim, -1)
        with _MatmulPrecision(cfg.role_kv_matmul_precision):
            if _projection_kernel_fits(dim, q_factor.shape[-1]):
                q_feat, _ = K.role_projection(q, q_factor, "row")
            else:
                q_feat = torch.bmm(q.float(), q_factor)
                q_feat = (q_feat / q_feat.square().mean(dim=2, keepdim=True).sqrt().clamp_min(1e-6)).contiguous()
            if q_init_features is None and warm:
                qi = torch.bmm(self.q_centroids, q_factor)
                q_init_features = qi / qi.square().mean(dim=2, keepdim=True).sqrt().clamp_min(1e-6)
        if q_init_features is None:
            idx = (self.init_indices[1] if self.init_indices is not None
                   else _init_indices(bh, tokens, cfg.num_q_centroids, cfg.kmeans_init_seed + 1, dev))
            q_init_features = torch.gather(q_feat, 1, idx.unsqueeze(-1).expand(-1, -1, q_feat.shape[-1]))
        q_labels, _qc, q_sizes, q_off, q_order, q_it = K.kmeans_lloyd(q_feat, q_init_features, iters, cfg.kmeans_tol,
                                                                     precision=cfg.kmeans_precision)
        q_cent, q_perm = K.centroid_means(q, q_order, q_off, cfg.num_q_centroids, self.q_centroids, permute=True)
        self.q_centroids = q_cent

        # Selector scores, budgets and the cluster-pair map (n8_v6.py:957-1112).
        if group > 1:
            k_cent_rt = k_cent.view(batch, kv_heads, -1, dim).repeat_interleave(group, dim=1).reshape(bh, -1, dim)
            v_cent_rt = v_cent.view(batch, kv_heads, -1, dim).repeat_interleave(group, dim=1).reshape(bh, -1, dim)
        else:
            k_cent_rt, v_cent_rt = k_cent, v_cent
        if cfg.selector_policy == "svg_ear_value":  # n8_v6.py:984-998 (no Jensen term)
            sk, sv = k_perm, v_perm
            if group > 1 and cfg.grouped_svg_ear_router:
                # n8_v6.py:936-971: every query head of a group is scored
                # against the group's native (first-head) sorted K/V.
                t = k_perm.shape[1]
                sk = k_perm.view(batch, heads, t, dim)[:, ::group].repeat_interleave(group, dim=1).reshape(bh, t, dim)
                sv = v_perm.view(batch, heads, t, dim)[:, ::group].repeat_interleave(group, dim=1).reshape(bh, t, dim)
            scores = K.svg_ear_value_scores(q_cent, sk, sv, k_cent_rt, v_cent_rt, k_off)
        else:  # attention_mass, n8_v6.py:971-983
            scores = K.attention_mass_scores(q_cent, k_perm, k_off)
        total_keys = int(total_key_tokens) if total_key_tokens is not None else tokens
        if total_keys < tokens or always_attended_keys < 0 or always_attended_keys > total_keys:
            raise ValueError(
                f"Invalid key accounting: video={tokens}, total={total_keys}, always={always_attended_keys}."
            )
        if cfg.selector_budget_mode == "fixed_density":
            base_total_density = max(0.0, cfg.target_density - cfg.probe_rows / float(tokens))
            budget = max(0, int(math.ceil(base_total_density * total_keys)) - int(always_attended_keys))
            budgets = torch.full((bh, cfg.num_q_centroids), budget, device=dev, dtype=torch.int32)
            base_density = budget / float(tokens)
        else:
            budgets = _svg_top_p_key_budgets(q_cent, k_cent_rt, k_sizes, cfg.svg_ear_top_p)
            budgets = budgets.clamp(min=int(math.ceil(cfg.adaptive_budget_min_density * tokens)),
                                    max=int(math.floor(cfg.adaptive_budget_max_density * tokens))).to(torch.int32)
            pair = (budgets.long() * q_sizes.long()).sum(dim=1).float() / float(tokens * tokens)
            # A 0-dim device tensor: read on the host only when the caller asks
            # (the reference synchronises here, n8_v6.py:1057-1060).
            base_density = pair.mean()
        routed, sel_ids, sel_counts = K.select_budget(scores, k_sizes, budgets)
        route = N8V6Route(
            q_labels=q_labels, k_labels=k_labels, q_cluster_sizes=q_sizes, k_cluster_sizes=k_sizes,
            video_dynamic_map=routed[:, 1:, 1:], q_role_features=q_feat,
            k_permuted=k_perm.view(batch, heads, -1, dim), v_permuted=v_perm.view(batch, heads, -1, dim),
            k_sorted_indices=k_order, base_video_density=base_density, q_kmeans_iters=iters, k_kmeans_iters=iters,
            permuted_includes_suffix=use_full, q_sorted_indices=q_order, q_permuted=q_perm, q_offsets=q_off,
            k_offsets=k_off, selected_ids=sel_ids, selected_counts=sel_counts, scores=scores, budgets=budgets,
            extras={"q_iters_done": q_it, "k_iters_done": k_it, "routed": routed},
        )
        self.route_call_index += 1
        return route

    # -- repair --------------------------------------------------------------
    def probe_rows(self, route: N8V6Route):
        """Probe rows and weights of ``route`` (selected once, cached on the route;
        ``residual_repair.py:118-260``)."""
        cfg = self.config
        if route.probe_rows is not None and route.probe_weights is not None:
            return route.probe_rows, route.probe_weights
        if cfg.probe_selection_policy == "first_token_largest_groups":
            rows, weights = select_first_token_largest_groups(route.q_role_features, route.q_labels,
                                                              cfg.num_q_centroids, cfg.probe_rows)
        else:
            rows, weights = select_role_equal_probes(route.q_role_features, route.q_labels, cfg.num_q_centroids,
                                                     cfg.probe_rows, order=route.q_sorted_indices,
                                                     offsets=route.q_offsets)
        route.probe_rows, route.probe_weights = rows, weights
        return rows, weights

    def fit_repair(self, base_probe, dense, weights, tokens: int, route: N8V6Route):
        """Fit the repair state from the probe rows' sparse output ``base_probe``
        and exact rows ``dense`` ([BH,M,D]); per-head recovery of a non-finite fit
        (``n8_v6.py:1244-1377``).  Returns ``(state, info)``."""
        cfg = self.config
        count, dim = int(base_probe.shape[1]), int(base_probe.shape[2])
        y_fit = dense.float() - base_probe.float()
        rank = min(cfg.repair_rank, count, dim)
        state = fit_reduced_rank_residual(base_probe.float(), y_fit, weights, rank, cfg.repair_ridge)
        state, self.repair_recovery_mask, policy = recover_nonfinite_rrr_state(state, self.repair_state_current)
        self.repair_state_current = state
        info = {
            "probe_rows": count,
            "probe_selection_policy": cfg.probe_selection_policy,
            "repair_rank": rank,
            "repair_feature_dim": dim,
            "repair_features": cfg.repair_features,
            "repair_basis_source": cfg.repair_basis_source,
            "repair_backend": "sparsepr_b200",
            "repair_recovery_policy": policy,
            "effective_video_density": _clamp_density(route.base_video_density + count / float(tokens)),
        }
        return state, info

    def fused_repair_supported(self, route: N8V6Route, dim: int) -> bool:
        """Whether the repair can run inside the attention epilogue
        (``spr_block_sparse_attn`` with a repair state): rank 16, d = 128,
        at most 128 probes and 1024 key clusters, output features, no norm cap."""
        cfg = self.config
        count = min(max(1, int(cfg.probe_rows)), int(route.q_labels.shape[1]))
        return (dim == 128 and min(cfg.repair_rank, count, dim) == 16 and count <= 128
                and route.k_offsets is not None and route.k_offsets.shape[-1] - 1 <= 1024
                and cfg.repair_norm_cap == 0.0 and cfg.repair_features == "output"
                and "routed" in route.extras and not route.permuted_includes_suffix)

    def repair(self, base_video, q_video, k_full, v_full, route: N8V6Route):
        """Probe-fitted residual repair of video rows (``n8_v6.py:1174-1444``).

        ``base_video`` [B,H,N,D] is the sparse attention output in the
        original token order; returns ``(corrected, info)``.
        """
        batch, heads, tokens, dim = base_video.shape
        bh = batch * heads
        cfg = self.config
        if cfg.repair_norm_cap > 0.0 or cfg.repair_features != "output":
            raise NotImplementedError("sparsepr_b200 repair implements output features without a norm cap.")
        base = base_video.to(torch.bfloat16).contiguous().view(bh, tokens, dim)
        rows, weights = self.probe_rows(route)
        q = q_video.to(torch.bfloat16).contiguous().view(bh, tokens, dim)
        kf = k_full.to(torch.bfloat16).contiguous().view(bh, -1, dim)
        vf = v_full.to(torch.bfloat16).contiguous().view(bh, -1, dim)
        gidx = rows.unsqueeze(2).expand(-1, -1, dim)
        dense = K.dense_attention_rows(torch.gather(q, 1, gidx), kf, vf)
        base_probe = torch.gather(base, 1, gidx)
        state, info = self.fit_repair(base_probe, dense, weights, tokens, route)
        corrected = K.repair_apply(base, state, cfg.repair_alpha, rows, dense)
        return corrected.view(batch, heads, tokens, dim), info
