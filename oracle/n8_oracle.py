"""CPU restatement of the SparsePR N8-V6 attention path (test oracle).

Test infrastructure only: imported by ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline legs, never by the product package.

All arithmetic is fp32 on the CPU (float64 where noted), following the
reference's own CPU branches where it has them and restating its Triton
kernels where it does not.  Reference paths are relative to the SparsePR
project root.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

__all__ = [
    "warm_subspace_metric_factor",
    "svg_ear_value_error_scores",
    "wan_qkv_norm_rope_layout",
    "euclid_assign",
    "assign_margin",
    "centroid_update",
    "batch_kmeans_euclid",
    "stable_label_order",
    "cluster_offsets",
    "original_centroids",
    "permute_rows",
    "inverse_permute_rows",
    "attention_mass_scores",
    "select_budget",
    "compact_selected",
    "fixed_density_budget",
    "svg_top_p_key_budgets",
    "block_sparse_attention",
    "dense_attention_rows",
    "select_role_equal_probes",
    "fit_reduced_rank_residual",
    "repair_apply",
    "deterministic_token_sample",
    "key_metric_from_queries",
    "query_metric_from_key_centroids",
    "metric_factor",
    "random_init_indices",
    "OracleRoute",
    "oracle_route",
    "OracleCore",
    "oracle_repair",
    "oracle_sparse_attention",
    "kept_pairs",
]


# ----------------------------------------------------------------------------
# (a5) Lloyd k-means
# ----------------------------------------------------------------------------

def euclid_assign(x: torch.Tensor, centroids: torch.Tensor) -> torch.Tensor:
    """Nearest centroid per point, ties to the lowest index.

    Follows ``flash_kmeans/assign_euclid_triton.py:803-917``
    (``dist = max(x_sq + c_sq - 2 x.c, 0)``, strict ``<`` across centroid
    tiles, ``tl.argmin`` inside a tile) and the torch fallback
    ``flash_kmeans/torch_fallback.py:4-53`` (``torch.argmin`` = first index).
    Distances in fp32 from the stored values.  x: [B,N,D], c: [B,K,D] ->
    int64 [B,N].
    """
    xf = x.float()
    cf = centroids.float()
    x_sq = (xf * xf).sum(-1)
    c_sq = (cf * cf).sum(-1)
    dist = x_sq.unsqueeze(-1) + c_sq.unsqueeze(-2) - 2.0 * torch.bmm(xf, cf.transpose(1, 2))
    dist = dist.clamp_min(0.0)
    return torch.argmin(dist, dim=-1)


def assign_margin(x: torch.Tensor, centroids: torch.Tensor) -> torch.Tensor:
    """Gap between the best and second-best squared distance, in float64.

    Test helper: points whose gap is below an fp32 rounding bound are
    "near ties" on which two correct fp32 implementations may disagree.
    """
    xd = x.double()
    cd = centroids.double()
    dist = (xd * xd).sum(-1, keepdim=True) + (cd * cd).sum(-1).unsqueeze(1) - 2 * torch.bmm(xd, cd.transpose(1, 2))
    top2 = torch.topk(dist, 2, dim=-1, largest=False).values
    return top2[..., 1] - top2[..., 0]


def centroid_update(x: torch.Tensor, labels: torch.Tensor, old: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Cluster means; an empty cluster keeps its old centroid.

    Follows ``flash_kmeans/torch_fallback.py:73-109`` and the sorted-run
    Triton update ``flash_kmeans/centroid_update_triton.py:316-386``
    (sums, ``counts.clamp(min=1)``, ``where(empty, old, mean)``); sums in
    float64, result fp32.  Returns (centroids fp32 [B,K,D], sizes int64 [B,K]).
    """
    b, n, d = x.shape
    k = old.shape[1]
    sums = torch.zeros((b, k, d), dtype=torch.float64)
    sums.scatter_add_(1, labels.long().unsqueeze(-1).expand(-1, -1, d), x.double())
    sizes = torch.zeros((b, k), dtype=torch.int64)
    sizes.scatter_add_(1, labels.long(), torch.ones_like(labels, dtype=torch.int64))
    means = (sums / sizes.clamp_min(1).unsqueeze(-1).double()).float()
    means = torch.where(sizes.unsqueeze(-1) > 0, means, old.float())
    return means, sizes


def batch_kmeans_euclid(
    x: torch.Tensor,
    n_clusters: int,
    max_iters: int,
    tol: float,
    init_centroids: torch.Tensor,
    *,
    centroid_dtype: torch.dtype | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, int]:
    """Batched Lloyd iterations with the reference's loop contract.

    Follows ``src/sparsepr/kmeans_utils.py:1281-1369`` and
    ``flash_kmeans/kmeans_triton_impl.py:55-115``: each iteration assigns
    against the current centroids, recomputes means, measures the max L2
    centroid shift, stops when ``shift < tol`` (keeping the pre-update
    centroids) and otherwise adopts the new centroids.  Returns
    ``(labels int64 [B,N], centroids [B,K,D], sizes int64 [B,K], iters)``;
    labels and sizes belong to the last assignment.

    ``centroid_dtype`` mirrors the standalone flash_kmeans path, which rounds
    the updated centroids to the input dtype every iteration
    (``centroid_update_triton.py:385``).
    """
    if max_iters < 1:
        raise ValueError("max_iters must be >= 1")
    centroids = init_centroids.float().clone()
    if centroid_dtype is not None:
        centroids = centroids.to(centroid_dtype).float()
    labels = sizes = None
    it = 0
    for it in range(max_iters):
        labels = euclid_assign(x, centroids)
        new, sizes = centroid_update(x, labels, centroids)
        if centroid_dtype is not None:
            new = new.to(centroid_dtype).float()
        shift = (new - centroids).norm(dim=-1).max()
        if shift < tol:
            break
        centroids = new
    return labels, centroids, sizes, it + 1


# ----------------------------------------------------------------------------
# (a6, a7) label order, centroid means, permute
# ----------------------------------------------------------------------------

def stable_label_order(labels: torch.Tensor) -> torch.Tensor:
    """Token order sorted by cluster label, ties by token index.

    The reference uses ``torch.argsort(labels)`` (``n8_v6.py:905``,
    ``wan22.py:2031``), which does not promise stability; within a cluster the
    order only permutes rows of one key/query block, so the build and this
    oracle both fix it to ascending token index.
    """
    return torch.argsort(labels.long(), dim=-1, stable=True)


def cluster_offsets(sizes: torch.Tensor) -> torch.Tensor:
    """Exclusive prefix sum of cluster sizes, [B,K] -> [B,K+1]
    (``svg_ear.py:432-441``)."""
    z = torch.zeros((sizes.shape[0], 1), dtype=torch.int64)
    return torch.cat((z, sizes.long().cumsum(1)), dim=1)


def original_centroids(x: torch.Tensor, labels: torch.Tensor, sizes: torch.Tensor,
                       fallback: torch.Tensor | None = None) -> torch.Tensor:
    """Mean of the original-space rows per label, fp32; empty clusters take
    ``fallback`` when given, else zero.  ``models/cosmos3/operator_kmeans.py:609-642``."""
    b, n, d = x.shape
    k = sizes.shape[1]
    sums = torch.zeros((b, k, d), dtype=torch.float64)
    sums.scatter_add_(1, labels.long().unsqueeze(-1).expand(-1, -1, d), x.double())
    means = (sums / sizes.clamp_min(1).unsqueeze(-1).double()).float()
    if fallback is not None:
        means = torch.where(sizes.unsqueeze(-1) > 0, means, fallback.float())
    return means


def permute_rows(x: torch.Tensor, order: torch.Tensor) -> torch.Tensor:
    """``y[:, s] = x[:, order[:, s]]`` for [BH,N,D] (``kmeans_utils.py:1674-1684``)."""
    return torch.gather(x, 1, order.long().unsqueeze(-1).expand(-1, -1, x.shape[-1]))


def inverse_permute_rows(y: torch.Tensor, order: torch.Tensor) -> torch.Tensor:
    """``x[:, order[:, s]] = y[:, s]`` (``kmeans_utils.py:1687-1695``)."""
    out = torch.empty_like(y)
    out.scatter_(1, order.long().unsqueeze(-1).expand(-1, -1, y.shape[-1]), y)
    return out


# ----------------------------------------------------------------------------
# (a8) selector scores, (a9) budgets, (a10) selector
# ----------------------------------------------------------------------------

def attention_mass_scores(q_centroids: torch.Tensor, k_sorted: torch.Tensor,
                          k_sizes: torch.Tensor) -> torch.Tensor:
    """``score[q, c] = log sum_{t in cluster c} exp(q_c . k_t / sqrt(D))``.

    Restates ``src/sparsepr/kernels/triton/svg_ear.py:7-92`` (wrapper
    372-450): keys are the cluster-sorted K rows, cluster ``c`` spans
    ``offsets[c]:offsets[c+1]``; an empty cluster scores ``-inf``.
    q_centroids [BH,Cq,D] fp32, k_sorted [BH,N,D] -> fp32 [BH,Cq,Ck].
    """
    bh, cq, d = q_centroids.shape
    ck = k_sizes.shape[1]
    logits = torch.bmm(q_centroids.float(), k_sorted.float().transpose(1, 2)) / math.sqrt(d)
    out = torch.full((bh, cq, ck), float("-inf"), dtype=torch.float32)
    for h in range(bh):
        seg = torch.repeat_interleave(torch.arange(ck), k_sizes[h].long()).unsqueeze(0).expand(cq, -1)
        m = torch.full((cq, ck), float("-inf"), dtype=torch.float32)
        m.scatter_reduce_(1, seg, logits[h], reduce="amax", include_self=True)
        e = torch.exp(logits[h] - m.gather(1, seg))
        s = torch.zeros((cq, ck), dtype=torch.float32)
        s.scatter_add_(1, seg, e)
        val = torch.log(s.clamp_min(1e-30)) + m
        out[h] = torch.where((k_sizes[h] > 0).unsqueeze(0), val, torch.full_like(val, float("-inf")))
    return out


def fixed_density_budget(target_density: float, probe_rows: int, tokens: int,
                         total_keys: int, always_attended: int) -> int:
    """Per-query-cluster key budget in fixed-density mode (``n8_v6.py:1026-1039``)."""
    base_total_density = max(0.0, target_density - probe_rows / float(tokens))
    target_keys = int(math.ceil(base_total_density * total_keys))
    return max(0, target_keys - int(always_attended))


def svg_top_p_key_budgets(q_centroids, k_centroids, k_sizes, top_p: float) -> torch.Tensor:
    """SVG2-style cumulative-mass budgets (``n8_v6.py:181-230``)."""
    dim = q_centroids.shape[2]
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


def select_budget(scores: torch.Tensor, k_sizes: torch.Tensor,
                  budgets: torch.Tensor) -> torch.Tensor:
    """Budgeted cluster selection -> routed map ``[BH, Cq+1, Ck+1]`` bool.

    Follows the CUDA-path rule of ``kernels/triton/selector_budget.py:10-54``
    (also ``kernels/n8_ext/csrc/n8_ops.cu:271-322``): order key clusters by
    descending score, keep the positive-size prefix whose cumulative size is
    ``<= budget``, then add the first crossing cluster when ``budget > 0``,
    the kept cost is below the budget and a positive cluster remains.  Row 0
    and column 0 are header entries (column 0 True for every row, row 0 False
    elsewhere).  Ties in score go to the lower cluster index (stable sort);
    the reference's ``torch.argsort`` leaves that order unspecified.
    """
    bh, cq, ck = scores.shape
    order = torch.argsort(-scores.float(), dim=2, stable=True)
    costs = torch.gather(k_sizes.long().unsqueeze(1).expand(-1, cq, -1), 2, order)
    positive = costs > 0
    cum = torch.where(positive, costs, 0).cumsum(dim=2)
    b = budgets.long().unsqueeze(2)
    keep = positive & (cum <= b)
    sel_cost = torch.where(keep, costs, 0).sum(dim=2)
    sel_count = keep.long().sum(dim=2)
    valid_count = positive.long().sum(dim=2)
    need = (budgets.long() > 0) & (sel_cost < budgets.long()) & (sel_count < valid_count)
    pos = torch.arange(ck).view(1, 1, ck)
    keep = keep | ((pos == sel_count.unsqueeze(2)) & need.unsqueeze(2))
    selected = torch.zeros((bh, cq, ck), dtype=torch.bool)
    selected.scatter_(2, order, keep)
    routed = torch.zeros((bh, cq + 1, ck + 1), dtype=torch.bool)
    routed[:, :, 0] = True
    routed[:, 1:, 1:] = selected
    return routed


def compact_selected(mask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Ascending selected cluster ids per row and their count
    (``kernels/n8_ext/csrc/n8_ops.cu:324-355``).  mask [..., Ck] bool ->
    (ids int32 [..., Ck] padded with -1, counts int32 [...])."""
    ck = mask.shape[-1]
    idx = torch.arange(ck).expand(mask.shape)
    key = torch.where(mask, idx, ck + idx)
    ids = torch.sort(key, dim=-1).values
    ids = torch.where(ids < ck, ids, torch.full_like(ids, -1)).to(torch.int32)
    return ids, mask.sum(-1).to(torch.int32)


# ----------------------------------------------------------------------------
# (a11) block-sparse attention, (a13) dense probe rows
# ----------------------------------------------------------------------------

def block_sparse_attention(q_perm, k_perm, v_perm, mask, q_sizes, k_sizes) -> torch.Tensor:
    """softmax(Q K^T / sqrt(D)) V restricted to kept (q-cluster, k-cluster) blocks.

    Same result as ``src/sparsepr/kmeans_utils.py:1748-1841``
    (``dynamic_block_sparse_fwd_torch``), vectorised per query cluster: a row
    whose cluster keeps no non-empty key cluster outputs zeros.  Inputs are
    cluster-sorted [BH,N,D]; fp32 math, output in the input dtype.
    mask [BH,Cq,Ck] bool (header row/col removed).
    """
    bh, n, d = q_perm.shape
    out = torch.zeros((bh, n, d), dtype=torch.float32)
    qo = cluster_offsets(q_sizes)
    scale = d ** -0.5
    for h in range(bh):
        qh, kh, vh = q_perm[h].float(), k_perm[h].float(), v_perm[h].float()
        seg = torch.repeat_interleave(torch.arange(k_sizes.shape[1]), k_sizes[h].long())
        for c in range(q_sizes.shape[1]):
            a, b = int(qo[h, c]), int(qo[h, c + 1])
            if a == b:
                continue
            keys = mask[h, c][seg]
            if not bool(keys.any()):
                continue
            s = qh[a:b] @ kh[keys].T * scale
            out[h, a:b] = torch.softmax(s, dim=-1) @ vh[keys]
    return out.to(q_perm.dtype)


def dense_attention_rows(q_rows, k, v) -> torch.Tensor:
    """Exact attention of selected query rows against all keys, fp32 math
    (``n8_v6.py:1234-1243`` uses SDPA).  [BH,M,D] x [BH,N,D] -> [BH,M,D] in q dtype."""
    d = q_rows.shape[-1]
    s = torch.bmm(q_rows.float(), k.float().transpose(1, 2)) * d ** -0.5
    return torch.bmm(torch.softmax(s, -1), v.float()).to(q_rows.dtype)


def kept_pairs(mask, q_sizes, k_sizes) -> int:
    """Selected (query, key) token pairs, the reference FLOP audit
    (``src/sparsepr/adapters/wan22.py:2044-2051``)."""
    sel_keys = (mask.long() * k_sizes.long().unsqueeze(1)).sum(-1)
    return int((sel_keys * q_sizes.long()).sum())


# ----------------------------------------------------------------------------
# (a12) probes, (a14) RRR fit, (a15) repair apply
# ----------------------------------------------------------------------------

def select_role_equal_probes(role_features, role_labels, num_clusters: int, rows: int):
    """One representative per largest role group, with group-size weights.

    Restates ``models/cosmos3/residual_repair.py:118-208``: per group the
    token closest (squared L2, fp32) to the group's feature mean, lowest token
    index on ties; groups ordered by descending size (stable); weight =
    group size / sampled count, normalised to mean 1.
    Returns (rows int64 [BH,M], weights fp32 [BH,M]).
    """
    bh, n, r = role_features.shape
    count = min(max(1, int(rows)), n)
    if count > num_clusters:
        raise RuntimeError(f"rows={count} must be <= clusters={num_clusters}")
    labels = role_labels.long()
    feats = role_features.float()
    sizes = torch.zeros((bh, num_clusters), dtype=torch.long)
    sizes.scatter_add_(1, labels, torch.ones_like(labels))
    sums = torch.zeros((bh, num_clusters, r), dtype=torch.float32)
    sums.scatter_add_(1, labels.unsqueeze(2).expand(-1, -1, r), feats)
    centers = sums / sizes.clamp_min(1).unsqueeze(2)
    dist = (feats - torch.gather(centers, 1, labels.unsqueeze(2).expand(-1, -1, r))).square().sum(2)
    best = torch.full((bh, num_clusters), float("inf"))
    best.scatter_reduce_(1, labels, dist, reduce="amin", include_self=True)
    tok = torch.arange(n).view(1, -1).expand(bh, -1)
    cand = torch.where(dist == torch.gather(best, 1, labels), tok, torch.full_like(tok, n))
    best_idx = torch.full((bh, num_clusters), n, dtype=torch.long)
    best_idx.scatter_reduce_(1, labels, cand, reduce="amin", include_self=True)
    order = torch.argsort(sizes, dim=1, descending=True, stable=True)
    sel = torch.gather(best_idx, 1, order)[:, :count]
    sel = torch.where(sel < n, sel, tok[:, :count])
    sel_labels = torch.gather(labels, 1, sel)
    sampled = torch.zeros_like(sizes)
    sampled.scatter_add_(1, sel_labels, torch.ones_like(sel_labels))
    gw = sizes.float() / sampled.clamp_min(1).float()
    w = torch.gather(gw, 1, sel_labels)
    w = w / w.mean(dim=1, keepdim=True).clamp_min(1e-20)
    return sel, w


def fit_reduced_rank_residual(x_fit, y_fit, weights, rank: int, ridge: float):
    """Weighted ridge reduced-rank regression, dual-Cholesky form, exact basis.

    Restates ``models/cosmos3/residual_repair.py:317-465`` on the path N8
    takes (``fit_backend='dual_cholesky'``, ``output_basis_backend='skinny'``,
    ``basis_source='raw_residual'``, rows < features) with the CPU basis
    ``reduced_rank_output_basis(backend='eigh')`` (468-491), in fp32 with the
    reference's op sequence (a rank-deficient fit, e.g. 16 probes at rank 16,
    is ill-conditioned, so another precision gives another, equally valid,
    blow-up of the weakest basis direction).
    Returns (x_mean, x_scale, y_mean [BH,1,D], left [BH,P,r], basis [BH,D,r]) fp32.
    """
    x = x_fit.float()
    y = y_fit.float()
    w = weights.float().unsqueeze(2)
    w_sum = w.sum(dim=1, keepdim=True).clamp_min(1e-20)
    x_mean = (w * x).sum(dim=1, keepdim=True) / w_sum
    x_var = (w * (x - x_mean).square()).sum(dim=1, keepdim=True) / w_sum
    x_scale = x_var.sqrt().clamp_min(1e-5)
    y_mean = (w * y).sum(dim=1, keepdim=True) / w_sum
    xn = (x - x_mean) / x_scale
    sw = w.sqrt()
    xw = xn * sw
    yw = (y - y_mean) * sw
    m = x.shape[1]
    if m >= x.shape[2]:
        raise RuntimeError("oracle fit covers the rows < features regime only")
    gram = torch.bmm(xw, xw.transpose(1, 2))
    gram.diagonal(dim1=1, dim2=2).add_(float(ridge))
    chol, _info = torch.linalg.cholesky_ex(gram, check_errors=False)
    dual = torch.cholesky_solve(yw, chol)
    evals, evecs = torch.linalg.eigh(torch.bmm(yw, yw.transpose(1, 2)))
    evecs = evecs[:, :, -rank:]
    scales = evals[:, -rank:].clamp_min(1e-20).rsqrt().unsqueeze(1)
    basis = (torch.bmm(yw.transpose(1, 2), evecs) * scales).contiguous()
    left = torch.bmm(xw.transpose(1, 2), torch.bmm(dual, basis)).contiguous()
    return x_mean, x_scale, y_mean, left, basis


def repair_apply(base, state, alpha: float = 1.0, norm_cap: float = 0.0):
    """``base + alpha * ((((base - mu_x)/sigma_x) L) B^T + mu_y)`` (CPU branch
    ``n8_v6.py:1378-1394``); result in base dtype."""
    x_mean, x_scale, y_mean, left, basis = state
    corr = torch.bmm(torch.bmm((base.float() - x_mean) / x_scale, left), basis.transpose(1, 2)) + y_mean
    if norm_cap > 0.0:
        bn = torch.linalg.vector_norm(base.float(), dim=2, keepdim=True)
        cn = torch.linalg.vector_norm(corr, dim=2, keepdim=True)
        corr = corr * (norm_cap * bn / cn.clamp_min(1e-20)).clamp_max(1.0)
    return base + alpha * corr.to(base.dtype)


# ----------------------------------------------------------------------------
# (a3, a4) role metrics, factors, projections
# ----------------------------------------------------------------------------

def deterministic_token_sample(x, sample_tokens: int):
    """Evenly spaced token subset (``operator_kmeans.py:52-59``)."""
    n = x.shape[1]
    if sample_tokens <= 0 or sample_tokens >= n:
        return x
    pos = torch.linspace(0, n - 1, steps=sample_tokens)
    return x[:, pos.round().long().unique(sorted=True)]


def key_metric_from_queries(q, sample_tokens: int):
    """Uncentered fp32 covariance of sampled queries (``operator_kmeans.py:491-493, 62-91``)."""
    s = deterministic_token_sample(q, sample_tokens).float()
    return torch.bmm(s.transpose(1, 2), s) / max(int(s.shape[1]), 1)


def query_metric_from_key_centroids(centroids, sizes):
    """Centered metric of non-empty K centroids (``operator_kmeans.py:514-529``)."""
    valid = (sizes > 0).float()
    count = valid.sum(1).clamp_min(1.0)
    mean = (centroids.float() * valid.unsqueeze(-1)).sum(1) / count.unsqueeze(-1)
    cen = (centroids.float() - mean.unsqueeze(1)) * valid.unsqueeze(-1)
    metric = torch.bmm(cen.transpose(1, 2), cen) / count.view(-1, 1, 1)
    return metric / float(centroids.shape[-1])


def metric_factor(metric, rank: int):
    """Top-``rank`` eigenvectors scaled by sqrt(eigenvalue / mean) (``operator_kmeans.py:94-151``)."""
    m = metric.float()
    m = 0.5 * (m + m.transpose(1, 2))
    evals, evecs = torch.linalg.eigh(m)
    evals = evals[:, -rank:].clamp_min(0.0)
    evecs = evecs[:, :, -rank:]
    norm = evals.mean(dim=1, keepdim=True).clamp_min(1e-12)
    return evecs * torch.sqrt(evals / norm).unsqueeze(1)


# ----------------------------------------------------------------------------
# (a2, a16, a17) composite route / repair / attention call
# ----------------------------------------------------------------------------

@dataclass
class OracleRoute:
    q_labels: torch.Tensor
    k_labels: torch.Tensor
    q_sizes: torch.Tensor
    k_sizes: torch.Tensor
    mask: torch.Tensor          # [BH,Cq,Ck] bool (header removed)
    q_features: torch.Tensor
    k_features: torch.Tensor
    q_centroids: torch.Tensor   # original space, fp32
    k_centroids: torch.Tensor
    v_centroids: torch.Tensor
    k_order: torch.Tensor
    q_order: torch.Tensor
    k_perm: torch.Tensor
    v_perm: torch.Tensor
    scores: torch.Tensor
    budgets: torch.Tensor
    q_iters: int
    k_iters: int


def random_init_indices(bh: int, n: int, k: int, seed: int) -> torch.Tensor:
    """Seeded random-sample initial centroid indices: ``randint(0, N, (BH, K))``
    like ``flash_kmeans/kmeans_triton_impl.py:89-96``, drawn from a CPU
    generator so every implementation sees the same indices."""
    g = torch.Generator().manual_seed(int(seed))
    return torch.randint(0, n, (bh, k), generator=g)


def _per_query_head(t, b, kvh, g):
    """Copy a per-KV-head tensor to each query head of its GQA group
    (``repeat_interleave`` over heads, ``n8_v6.py:762-834``)."""
    return t.reshape(b, kvh, *t.shape[1:]).repeat_interleave(g, dim=1).reshape(b * kvh * g, *t.shape[1:])


def oracle_route(q, k, v, cfg, *, k_init=None, q_init=None, init_seed: int = 0,
                 tol: float = 0.0, gqa_group_size: int = 1) -> OracleRoute:
    """Cold-start ``N8V6Core.route`` (``models/common/n8_v6.py:521-1172``) for
    the attention-mass or SVG-EAR value-error selector (``n8_v6.py:971-998``),
    fixed-density or top-p budgets, no text suffix.  ``cfg`` carries the ``N8V6Config`` fields used here.
    ``k_init``/``q_init`` are role-feature-space initial centroids; when
    omitted they are the rows at ``random_init_indices``.

    GQA (``gqa_group_size`` g > 1, ``n8_v6.py:549-567, 762-834, 936-971``):
    K/V are clustered on the first query head of each group with the key
    metric pooled over the group's g*N queries (g times the sample count,
    ``operator_kmeans.py:570-606``); the Q factor, K labels, sizes and
    centroids are then copied to every query head of the group, and each
    query head permutes its own K/V by the group's order.  The returned
    ``k_features`` stay per KV head."""
    b, h, n, d = q.shape
    g = int(gqa_group_size)
    if g <= 0 or h % g:
        raise ValueError(f"gqa_group_size must divide the query-head count; got H={h}, G={g}.")
    bh, kvh = b * h, h // g
    qf3, kf3, vf3 = (t.reshape(bh, n, d) for t in (q, k, v))
    kn3 = k[:, ::g].reshape(b * kvh, n, d)
    vn3 = v[:, ::g].reshape(b * kvh, n, d)
    k_factor = metric_factor(key_metric_from_queries(qf3.reshape(b * kvh, g * n, d), cfg.metric_sample_tokens * g),
                             cfg.role_k_rank)
    kfeat = torch.bmm(kn3.float(), k_factor)
    kscale = kfeat.square().mean(dim=(1, 2), keepdim=True).sqrt().clamp_min(1e-8)
    kfeat = kfeat / kscale
    if k_init is None:
        idx = random_init_indices(b * kvh, n, cfg.num_k_centroids, init_seed)
        k_init = torch.gather(kfeat, 1, idx.unsqueeze(-1).expand(-1, -1, kfeat.shape[-1]))
    k_labels, _, k_sizes, k_it = batch_kmeans_euclid(kfeat, cfg.num_k_centroids, cfg.kmeans_iter_init, tol, k_init)
    k_cent = original_centroids(kn3, k_labels, k_sizes)
    v_cent = original_centroids(vn3, k_labels, k_sizes)
    q_factor = metric_factor(query_metric_from_key_centroids(k_cent, k_sizes), cfg.role_q_rank)
    if g > 1:
        q_factor, k_labels, k_sizes, k_cent, v_cent = (_per_query_head(t, b, kvh, g)
                                                      for t in (q_factor, k_labels, k_sizes, k_cent, v_cent))
    qfeat = torch.bmm(qf3.float(), q_factor)
    qfeat = qfeat / qfeat.square().mean(dim=2, keepdim=True).sqrt().clamp_min(1e-6)
    if q_init is None:
        idx = random_init_indices(bh, n, cfg.num_q_centroids, init_seed + 1)
        q_init = torch.gather(qfeat, 1, idx.unsqueeze(-1).expand(-1, -1, qfeat.shape[-1]))
    q_labels, _, q_sizes, q_it = batch_kmeans_euclid(qfeat, cfg.num_q_centroids, cfg.kmeans_iter_init, tol, q_init)
    q_cent = original_centroids(qf3, q_labels, q_sizes)
    k_order = stable_label_order(k_labels)
    q_order = stable_label_order(q_labels)
    k_perm = permute_rows(kf3, k_order)
    v_perm = permute_rows(vf3, k_order)
    if getattr(cfg, "selector_policy", "attention_mass") == "svg_ear_value":
        sk, sv = k_perm, v_perm
        if g > 1 and getattr(cfg, "grouped_svg_ear_router", False):  # native K/V of each group
            sk = _per_query_head(k_perm.reshape(b, h, n, d)[:, ::g].reshape(b * kvh, n, d), b, kvh, g)
            sv = _per_query_head(v_perm.reshape(b, h, n, d)[:, ::g].reshape(b * kvh, n, d), b, kvh, g)
        scores = svg_ear_value_error_scores(q_cent, sk, sv, k_cent, v_cent, k_sizes)
    else:
        scores = attention_mass_scores(q_cent, k_perm, k_sizes)
    if cfg.selector_budget_mode == "fixed_density":
        budget = fixed_density_budget(cfg.target_density, cfg.probe_rows, n, n, 0)
        budgets = torch.full((bh, cfg.num_q_centroids), budget, dtype=torch.long)
    else:
        budgets = svg_top_p_key_budgets(q_cent, k_cent, k_sizes, cfg.svg_ear_top_p)
        budgets = budgets.clamp(min=int(math.ceil(cfg.adaptive_budget_min_density * n)),
                                max=int(math.floor(cfg.adaptive_budget_max_density * n)))
    routed = select_budget(scores, k_sizes, budgets)
    return OracleRoute(q_labels, k_labels, q_sizes, k_sizes, routed[:, 1:, 1:], qfeat, kfeat,
                       q_cent, k_cent, v_cent, k_order, q_order, k_perm, v_perm, scores, budgets, q_it, k_it)


class OracleCore:
    """Stateful ``N8V6Core.route`` across calls (``models/common/n8_v6.py:372-1172``),
    symmetric heads (no GQA), no text suffix, ``factor_refresh_every = 1``.

    The first call is :func:`oracle_route` (cold start, ``kmeans_iter_init``
    iterations from the rows at ``random_init_indices``).  Later calls are the
    reference's warm path:

    * role factors by warm subspace iteration from the previous bases
      (``n8_v6.py:478-519`` -> ``operator_kmeans.py:221-477``), a head whose
      warm solve fails keeping its previous factor and basis;
    * K initial centroids = previous original-space K centroids projected by
      the new K factor and divided by the new K feature scale
      (``n8_v6.py:686-697``); Q initial centroids = previous Q centroids
      projected by the new Q factor, row-RMS normalised (``n8_v6.py:779-783``);
    * ``kmeans_iter_step`` Lloyd iterations for both (``n8_v6.py:698``) with the
      k-means ``tol``;
    * original-space centroids with empty clusters keeping the previous ones
      (``n8_v6.py:734-741, 796``).
    """

    def __init__(self, cfg, *, init_seed: int = 0, tol: float = 1e-4):
        self.cfg = cfg
        self.init_seed = int(init_seed)
        self.tol = float(tol)
        self.state = None

    def route(self, q, k, v) -> OracleRoute:
        if self.state is None:
            r, self.state = _route(q, k, v, self.cfg, None, init_seed=self.init_seed, tol=self.tol)
        else:
            r, self.state = _route(q, k, v, self.cfg, self.state, tol=self.tol)
        return r


def _route(q, k, v, cfg, prev, *, init_seed: int = 0, tol: float = 0.0):
    """One call of :class:`OracleCore`: cold when ``prev`` is None, else warm from
    ``prev`` (dict of the previous call's centroids and factor states)."""
    b, h, n, d = q.shape
    bh = b * h
    q3, k3, v3 = (t.reshape(bh, n, d) for t in (q, k, v))
    if prev is None:
        r = oracle_route(q, k, v, cfg, init_seed=init_seed, tol=tol)
        kf = metric_factor(key_metric_from_queries(q3, cfg.metric_sample_tokens), cfg.role_k_rank)
        qf = metric_factor(query_metric_from_key_centroids(r.k_centroids, r.k_sizes), cfg.role_q_rank)
        return r, {"k_centroids": r.k_centroids, "v_centroids": r.v_centroids, "q_centroids": r.q_centroids,
                   "k_factor": kf, "k_basis": kf, "q_factor": qf, "q_basis": qf}
    warm = dict(power_iters=getattr(cfg, "factor_power_iters", 2),
                rayleigh_ridge=getattr(cfg, "factor_rayleigh_ridge", 1e-4),
                cholesky_qr_ridge=getattr(cfg, "factor_cholesky_qr_ridge", 1e-5))

    def updated(metric, basis, current, rank):
        f, st, bad = warm_subspace_metric_factor(metric, basis, rank, **warm)
        sel = bad[:, None, None]
        return torch.where(sel, current, f), torch.where(sel, basis, st)

    k_factor, k_basis = updated(key_metric_from_queries(q3, cfg.metric_sample_tokens), prev["k_basis"],
                                prev["k_factor"], cfg.role_k_rank)
    kfeat = torch.bmm(k3.float(), k_factor)
    kscale = kfeat.square().mean(dim=(1, 2), keepdim=True).sqrt().clamp_min(1e-8)
    kfeat = kfeat / kscale
    k_init = torch.bmm(prev["k_centroids"], k_factor) / kscale
    iters = cfg.kmeans_iter_step
    k_labels, _, k_sizes, k_it = batch_kmeans_euclid(kfeat, cfg.num_k_centroids, iters, tol, k_init)
    k_cent = original_centroids(k3, k_labels, k_sizes, prev["k_centroids"])
    v_cent = original_centroids(v3, k_labels, k_sizes, prev["v_centroids"])
    q_factor, q_basis = updated(query_metric_from_key_centroids(k_cent, k_sizes), prev["q_basis"],
                                prev["q_factor"], cfg.role_q_rank)
    qfeat = torch.bmm(q3.float(), q_factor)
    qfeat = qfeat / qfeat.square().mean(dim=2, keepdim=True).sqrt().clamp_min(1e-6)
    qi = torch.bmm(prev["q_centroids"], q_factor)
    q_init = qi / qi.square().mean(dim=2, keepdim=True).sqrt().clamp_min(1e-6)
    q_labels, _, q_sizes, q_it = batch_kmeans_euclid(qfeat, cfg.num_q_centroids, iters, tol, q_init)
    q_cent = original_centroids(q3, q_labels, q_sizes, prev["q_centroids"])
    k_order = stable_label_order(k_labels)
    q_order = stable_label_order(q_labels)
    k_perm = permute_rows(k3, k_order)
    v_perm = permute_rows(v3, k_order)
    if getattr(cfg, "selector_policy", "attention_mass") == "svg_ear_value":
        scores = svg_ear_value_error_scores(q_cent, k_perm, v_perm, k_cent, v_cent, k_sizes)
    else:
        scores = attention_mass_scores(q_cent, k_perm, k_sizes)
    if cfg.selector_budget_mode == "fixed_density":
        budget = fixed_density_budget(cfg.target_density, cfg.probe_rows, n, n, 0)
        budgets = torch.full((bh, cfg.num_q_centroids), budget, dtype=torch.long)
    else:
        budgets = svg_top_p_key_budgets(q_cent, k_cent, k_sizes, cfg.svg_ear_top_p)
        budgets = budgets.clamp(min=int(math.ceil(cfg.adaptive_budget_min_density * n)),
                                max=int(math.floor(cfg.adaptive_budget_max_density * n)))
    routed = select_budget(scores, k_sizes, budgets)
    r = OracleRoute(q_labels, k_labels, q_sizes, k_sizes, routed[:, 1:, 1:], qfeat, kfeat,
                    q_cent, k_cent, v_cent, k_order, q_order, k_perm, v_perm, scores, budgets, q_it, k_it)
    return r, {"k_centroids": k_cent, "v_centroids": v_cent, "q_centroids": q_cent,
               "k_factor": k_factor, "k_basis": k_basis, "q_factor": q_factor, "q_basis": q_basis}


def oracle_repair(base, q, k, v, route, cfg):
    """``N8V6Core.repair`` CPU branch (``n8_v6.py:1174-1444``) with output
    features and the exact-eigh basis.  base/q/k/v [BH,N,D]."""
    rows, weights = select_role_equal_probes(route.q_features, route.q_labels,
                                             cfg.num_q_centroids, cfg.probe_rows)
    d = q.shape[-1]
    gidx = rows.unsqueeze(2).expand(-1, -1, d)
    dense = dense_attention_rows(torch.gather(q, 1, gidx), k, v)
    base_probe = torch.gather(base.float(), 1, gidx)
    y_fit = dense.float() - base_probe
    rank = min(cfg.repair_rank, rows.shape[1], d)
    state = fit_reduced_rank_residual(base_probe, y_fit, weights, rank, cfg.repair_ridge)
    out = repair_apply(base, state, cfg.repair_alpha, cfg.repair_norm_cap)
    out.scatter_(1, gidx, dense.to(out.dtype))
    return out, state, rows, weights, dense


def oracle_sparse_attention(q, k, v, cfg, *, route=None, **route_kw):
    """``_sparse_n8_attention_bhld`` (``adapters/wan22.py:1945-2182``):
    route, Q permute, block-sparse attention, inverse permute, repair.
    q/k/v [B,H,N,D] -> (out [B,H,N,D], route, base [BH,N,D], repair pieces)."""
    b, h, n, d = q.shape
    bh = b * h
    if route is None:
        route = oracle_route(q, k, v, cfg, **route_kw)
    q3, k3, v3 = (t.reshape(bh, n, d) for t in (q, k, v))
    q_perm = permute_rows(q3, route.q_order)
    out_perm = block_sparse_attention(q_perm, route.k_perm, route.v_perm, route.mask,
                                      route.q_sizes, route.k_sizes)
    base = inverse_permute_rows(out_perm, route.q_order)
    out, state, rows, weights, dense = oracle_repair(base, q3, k3, v3, route, cfg)
    return out.view(b, h, n, d), route, base, (state, rows, weights, dense)


def wan_qkv_norm_rope_layout(q, k, v, q_weight, k_weight, freq_real, freq_imag, heads: int, epsilon: float):
    """CPU restatement of the reference's fused Wan producer kernel
    (``src/sparsepr/kernels/n8_ext/csrc/n8_ops.cu:16-105``, host 357-411).

    Per token row: mean of squares over all C channels in fp32, ``inv =
    1/sqrt(mean + eps)``; ``x * inv * w`` in fp32 rounded once to the model
    dtype (the kernel's order; Wan's torch path rounds before the weight);
    RoPE on channel pairs (2i, 2i+1) of each head, ``(a + ib)(fr + i fi)`` in
    fp32, rounded to the model dtype; layout [B,L,C] -> [B,H,L,D].  V is only
    re-laid out.
    """
    b, l, c = q.shape
    hd = c // heads
    dt = q.dtype

    def norm_rope(x, w):
        xf = x.float()
        inv = torch.rsqrt(xf.square().mean(dim=-1, keepdim=True) + epsilon)
        y = (xf * inv * w.float()).to(dt).float().view(b, l, heads, hd // 2, 2)
        a, bb = y[..., 0], y[..., 1]
        fr = freq_real.float().view(1, l, 1, hd // 2)
        fi = freq_imag.float().view(1, l, 1, hd // 2)
        out = torch.stack((a * fr - bb * fi, a * fi + bb * fr), dim=-1).to(dt)
        return out.view(b, l, heads, hd).permute(0, 2, 1, 3).contiguous()

    vo = v.view(b, l, heads, hd).permute(0, 2, 1, 3).contiguous()
    return norm_rope(q, q_weight), norm_rope(k, k_weight), vo


def svg_ear_value_error_scores(qc, k_sorted, v_sorted, k_centroids, v_centroids, k_sizes):
    """SVG-EAR value-error selector scores (``kernels/triton/svg_ear.py:95-193``,
    wrapper 453-531, no Jensen term as the route calls it, ``n8_v6.py:984-998``).

    For query centroid c and key cluster j with tokens t:
        a = exp(q_c . kbar_j / sqrt(D)),  b_t = exp(q_c . k_t / sqrt(D))
        score = log( (1/n_j) sum_t |a vbar_j - b_t v_t|^2 )
    (-inf for an empty cluster; the error is floored at 1e-30 before the log),
    evaluated here in float64 with a per-(c, j) max shift.
    """
    bh, cq, d = qc.shape
    ck = k_centroids.shape[1]
    off = cluster_offsets(k_sizes.long())
    scale = 1.0 / math.sqrt(d)
    out = torch.full((bh, cq, ck), float("-inf"), dtype=torch.float64)
    for b in range(bh):
        q = qc[b].double()
        for j in range(ck):
            s, e = int(off[b, j]), int(off[b, j + 1])
            if e <= s:
                continue
            kt = k_sorted[b, s:e].double()
            vt = v_sorted[b, s:e].double()
            cl = (q @ k_centroids[b, j].double()) * scale              # [cq]
            tl = (q @ kt.T) * scale                                     # [cq, nj]
            m = torch.maximum(cl, tl.max(dim=1).values)
            a = torch.exp(cl - m).unsqueeze(1)                          # [cq, 1]
            bt = torch.exp(tl - m.unsqueeze(1))                         # [cq, nj]
            vbar = v_centroids[b, j].double()
            err = (a * a * vbar.dot(vbar) + bt * bt * (vt * vt).sum(1) - 2 * a * bt * (vt @ vbar)).clamp_min(0)
            out[b, :, j] = torch.log((err.sum(1) / (e - s)).clamp_min(1e-30)) + 2 * m
    return out.float()


def warm_subspace_metric_factor(metric, previous, rank, *, power_iters=2, orthogonalization="each_cholesky_qr2",
                                rayleigh_ridge=1e-4, cholesky_qr_ridge=1e-5):
    """Warm role factor by subspace iteration with the Rayleigh-Cholesky Ritz
    step, restating ``operator_kmeans.py:221-477`` (Cholesky-QR 332-364,
    ridge fallback ``cholesky_with_device_fallback`` 154-218).  Returns
    ``(factor, basis, recovered)``."""
    m = metric.float()
    basis = previous.float()
    basis = basis / torch.linalg.vector_norm(basis, dim=1, keepdim=True).clamp_min(1e-12)
    recovered = torch.zeros(m.shape[0], dtype=torch.bool)

    def chol_qr(x, ridge):
        xn = x / torch.linalg.vector_norm(x, dim=1, keepdim=True).clamp_min(1e-12)
        g = torch.bmm(xn.transpose(1, 2), xn)
        g = 0.5 * (g + g.transpose(1, 2))
        jit = g.diagonal(dim1=1, dim2=2).mean(dim=1, keepdim=True).clamp_min(1e-12) * ridge
        g = g + torch.diag_embed(jit.expand(-1, g.shape[-1]))
        ch, info = torch.linalg.cholesky_ex(g)
        bad = info != 0
        ch = torch.where(bad[:, None, None], torch.eye(g.shape[-1]).expand_as(ch), ch)
        return torch.linalg.solve_triangular(ch, xn.transpose(1, 2), upper=False).transpose(1, 2), bad

    for it in range(power_iters):
        basis, bad = chol_qr(torch.bmm(m, basis), cholesky_qr_ridge)
        recovered |= bad
        if orthogonalization == "each_cholesky_qr2" and it == power_iters - 1:
            basis, bad = chol_qr(basis, max(cholesky_qr_ridge, 1e-5))
            recovered |= bad
    r = torch.bmm(basis.transpose(1, 2), torch.bmm(m, basis))
    r = 0.5 * (r + r.transpose(1, 2))
    norm = r.diagonal(dim1=1, dim2=2).mean(dim=1).clamp_min(1e-12)
    eye = torch.eye(r.shape[-1]).expand_as(r)
    prim, pinfo = torch.linalg.cholesky_ex(r + (norm * rayleigh_ridge)[:, None, None] * eye)
    fb, finfo = torch.linalg.cholesky_ex(r + (norm * max(1e-2, rayleigh_ridge))[:, None, None] * eye)
    use_p = (pinfo == 0)[:, None, None]
    use_f = (~use_p) & (finfo == 0)[:, None, None]
    chol = torch.where(use_p, prim, torch.where(use_f, fb, eye))
    recovered |= finfo != 0
    factor = torch.bmm(basis, chol) / torch.sqrt(norm)[:, None, None]
    recovered |= ~torch.isfinite(factor).all(dim=(1, 2)) | ~torch.isfinite(basis).all(dim=(1, 2))
    return factor, basis, recovered
