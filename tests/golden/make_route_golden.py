"""Two-call D=128 route fixture from the REFERENCE's own ``N8V6Core`` on the CPU.

    python tests/golden/make_route_golden.py /path/to/SparsePR

Runs the reference's ``N8V6Core.route`` twice on one core (a cold call, then
a warm call on the next step's inputs) with the same three CUDA-only shims as
``make_golden.py`` (torch k-means fallback with the reference's ``tol=1e-4``
and seeded cold-start rows, ``torch.gather`` permute, per-cluster logsumexp
attention-mass scores).  The warm call is the reference's own code
unchanged: warm subspace-iteration factors, projected previous centroids,
``kmeans_iter_step`` iterations.  D = 128, 2 heads, 1,536 tokens on a 6x16x16
grid, Cq = 32, Ck = 64, fixed density 0.3, attention-mass selector.

Output: ``tests/golden/route_d128_two_calls.pt`` with, per call, checksums of
the inputs (which ``inputs()`` regenerates), labels, sizes, the [BH,Cq,Ck]
map, iteration counts and original-space centroids.
"""

from __future__ import annotations

import math
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
SEEDS = {"k": 100, "q": 101}
GRID = (6, 16, 16)
CONFIG = dict(num_q_centroids=32, num_k_centroids=64, target_density=0.3, kmeans_iter_init=10, kmeans_iter_step=2,
              probe_rows=32, repair_rank=16, selector_policy="attention_mass", selector_budget_mode="fixed_density")


def inputs():
    """Step-1 inputs (smooth field + noise) and step-2 inputs (the same fields
    moved a little: 0.95 x step 1 + 0.25 x fresh noise), [1,2,N,128] fp32
    holding bf16-representable values (the attention path stores bf16)."""
    from sparsepr_b200.synthetic import synthetic_qkv

    q, k, v = synthetic_qkv(2, 128, GRID, dtype=torch.float32, seeds=(21, 22, 23))
    g = torch.Generator().manual_seed(24)
    step2 = tuple(0.95 * t + 0.25 * torch.randn(t.shape, generator=g) for t in (q, k, v))
    bf = lambda ts: tuple(t.to(torch.bfloat16).float() for t in ts)  # noqa: E731
    return bf((q, k, v)), bf(step2)


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "src"))
    sys.path.insert(0, REPO)
    from flash_kmeans.torch_fallback import batch_kmeans_Euclid_torch_native
    import sparsepr.models.common.n8_v6 as n8

    from sparsepr_b200.synthetic import random_init_indices

    calls = {"n": 0}

    def kmeans_shim(x, n_clusters, max_iters=100, tol=1e-4, init_centroids=None, verbose=False, backend=None):
        if init_centroids is None:
            role = "k" if calls["n"] % 2 == 0 else "q"
            idx = random_init_indices(x.shape[0], x.shape[1], n_clusters, SEEDS[role])
            init_centroids = torch.gather(x, 1, idx.unsqueeze(-1).expand(-1, -1, x.shape[-1]))
        calls["n"] += 1
        ids, cents, iters = batch_kmeans_Euclid_torch_native(
            x, n_clusters, max_iters=max_iters, tol=tol, init_centroids=init_centroids)
        ones = torch.ones_like(ids, dtype=torch.int64)
        sizes = torch.zeros((x.shape[0], n_clusters), dtype=torch.int64).scatter_add_(1, ids.long(), ones)
        return ids.long(), cents, sizes, iters

    def permute_shim(tensor, labels, dim, sorted_indices=None):
        idx = sorted_indices.long()
        g = idx.unsqueeze(-1).expand(*idx.shape, tensor.shape[-1]).reshape(tensor.shape)
        return torch.gather(tensor, dim, g), sorted_indices

    def scores_shim(*, qcentroids, k_sorted, kcluster_sizes, gqa_group, logical_tokens=None, **_):
        bh, cq, d = qcentroids.shape
        ck = kcluster_sizes.shape[1]
        out = torch.full((bh, cq, ck), float("-inf"))
        offs = torch.cat((torch.zeros(bh, 1, dtype=torch.long), kcluster_sizes.long().cumsum(1)), 1)
        for h in range(bh):
            for c in range(ck):
                a, b = int(offs[h, c]), int(offs[h, c + 1])
                if b > a:
                    lg = qcentroids[h].float() @ k_sorted[h, a:b].float().T / math.sqrt(d)
                    out[h, :, c] = torch.logsumexp(lg, dim=1)
        return out

    n8.batch_kmeans_Euclid = kmeans_shim
    n8.permute_tensor_by_labels_triton = permute_shim
    n8.attention_mass_scores_triton = scores_shim

    steps = inputs()
    core = n8.N8V6Core(n8.N8V6Config(compile_role_kv_projection=False, **CONFIG))
    out = {"config": dict(CONFIG, tol=1e-4, seed_k=SEEDS["k"], seed_q=SEEDS["q"], grid=GRID), "calls": []}
    for i, (q, k, v) in enumerate(steps):
        calls["n"] = 0
        route = core.route(q, k, v, total_key_tokens=q.shape[2])
        out["calls"].append({
            "input_sums": [float(t.double().sum()) for t in (q, k, v)],
            "q_labels": route.q_labels.to(torch.int16), "k_labels": route.k_labels.to(torch.int16),
            "q_sizes": route.q_cluster_sizes.clone(), "k_sizes": route.k_cluster_sizes.clone(),
            "mask": route.video_dynamic_map.clone(),
            "q_iters": int(route.q_kmeans_iters), "k_iters": int(route.k_kmeans_iters),
            "k_centroids": core.k_centroids.clone(), "v_centroids": core.v_centroids.clone(),
            "q_centroids": core.q_centroids.clone(),
        })
        print("call", i, "k_iters", route.k_kmeans_iters, "q_iters", route.q_kmeans_iters)
    torch.save(out, os.path.join(HERE, "route_d128_two_calls.pt"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_route_golden.py /path/to/SparsePR")
    main(sys.argv[1])
