"""Generate golden vectors by running the REFERENCE SparsePR code on the CPU.

Run in a container that has the reference checkout (it is never read at test
time):

    python tests/golden/make_golden.py /path/to/SparsePR

The reference's N8-V6 core (``src/sparsepr/models/common/n8_v6.py``) runs
unchanged on the CPU except for three CUDA-only calls, swapped for the
reference's own torch equivalents or a CPU restatement of the Triton math:

* ``batch_kmeans_Euclid`` -> ``flash_kmeans/torch_fallback.py``
  ``batch_kmeans_Euclid_torch_native`` (same assign/update/shift loop) with the
  reference's default ``tol=1e-4`` and sizes by ``scatter_add`` as in
  ``kmeans_utils.py:1119-1121``; cold-start centroids are the rows at a
  seeded ``randint`` instead of the global RNG.
* ``permute_tensor_by_labels_triton`` -> ``torch.gather`` by the sorted indices
  (``kmeans_utils.py:1674-1684``).
* ``attention_mass_scores_triton`` -> per-cluster ``logsumexp`` of
  ``q_c . k / sqrt(D)`` (``svg_ear.py:7-92``).

The attention step is the reference's ``dynamic_block_sparse_fwd_torch``
(``kmeans_utils.py:1748-1841``) and ``apply_inverse_permutation``
(1687-1695); repair is ``N8V6Core.repair``'s CPU branch.  Output:
``tests/golden/config0_<mode>.pt``.

A GQA case (4 query heads, ``gqa_group_size=2``, K/V heads that differ
within a group) records the reference route's labels, sizes, K/V centroids,
Q factor features and map: ``tests/golden/config0_gqa.pt``.

An SVG-EAR value-error case (``selector_policy="svg_ear_value"``, D = 128, the
scorer's only width) runs the reference's own ``_svg_ear_value_error_kernel``
(``svg_ear.py:95-193``) through Triton's CPU interpreter (``TRITON_INTERPRET=1``,
launched as its wrapper ``svg_ear_value_error_scores_triton`` launches it,
``svg_ear.py:453-531``) inside the route: ``tests/golden/config0_svg_value.pt``.
"""

from __future__ import annotations

import math
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def main(ref_root: str) -> None:
    os.environ["TRITON_INTERPRET"] = "1"  # only the SVG-EAR case runs a Triton kernel (on CPU)
    sys.path.insert(0, os.path.join(ref_root, "src"))
    sys.path.insert(0, REPO)
    from flash_kmeans.torch_fallback import batch_kmeans_Euclid_torch_native
    import sparsepr.models.common.n8_v6 as n8
    from sparsepr.kmeans_utils import apply_inverse_permutation, dynamic_block_sparse_fwd_torch

    from sparsepr_b200.synthetic import random_init_indices, synthetic_qkv

    seeds = {"k": 100, "q": 101}
    calls = {"n": 0}

    def kmeans_shim(x, n_clusters, max_iters=100, tol=1e-4, init_centroids=None, verbose=False, backend=None):
        if init_centroids is None:
            role = "k" if calls["n"] % 2 == 0 else "q"
            idx = random_init_indices(x.shape[0], x.shape[1], n_clusters, seeds[role])
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

    def svg_shim(*, qcentroids, k_sorted, v_sorted, kcentroids, vcentroids, kcluster_sizes, gqa_group,
                 block_q, block_n, logical_tokens=None, **_):
        import triton
        from sparsepr.kernels.triton.svg_ear import _svg_ear_value_error_kernel

        h, cq, d = qcentroids.shape
        ck = kcluster_sizes.shape[1]
        tokens = k_sorted.shape[1]
        off = torch.cat((torch.zeros(h, 1, dtype=torch.int32), kcluster_sizes.int().cumsum(1).int()), 1).contiguous()
        scores = torch.empty(h, cq, ck)
        bq = min(block_q, 16)
        _svg_ear_value_error_kernel[(triton.cdiv(cq, bq), ck, h)](
            qcentroids.float().contiguous(), k_sorted.contiguous(), v_sorted.contiguous(),
            kcentroids.float().contiguous(), vcentroids.float().contiguous(), kcentroids.float().contiguous(), off,
            scores, Q_CLUSTERS=cq, K_CLUSTERS=ck, TOKENS=tokens, SORTED_HEAD_STRIDE=tokens, DIM=d,
            GQA_GROUP=gqa_group, JENSEN_VAR_CAP=0.0, USE_JENSEN=False, BLOCK_Q=bq, BLOCK_N=min(block_n, 32))
        return scores

    n8.batch_kmeans_Euclid = kmeans_shim
    n8.svg_ear_value_error_scores_triton = svg_shim
    n8.permute_tensor_by_labels_triton = permute_shim
    n8.attention_mass_scores_triton = scores_shim

    q, k, v = synthetic_qkv(2, 64, (4, 8, 8), dtype=torch.float32)
    for mode in ("fixed_density", "svg_ear_top_p"):
        calls["n"] = 0
        cfg = n8.N8V6Config(
            num_q_centroids=16, num_k_centroids=32, target_density=0.25,
            kmeans_iter_init=8, kmeans_iter_step=2, probe_rows=16, repair_rank=16,
            selector_policy="attention_mass", selector_budget_mode=mode, svg_ear_top_p=0.25,
            compile_role_kv_projection=False,
        )
        core = n8.N8V6Core(cfg)
        route = core.route(q, k, v, total_key_tokens=q.shape[2])
        q3 = q.reshape(2, 256, 64)
        q_order = torch.argsort(route.q_labels, dim=-1, stable=True)
        q_perm = torch.gather(q3, 1, q_order.unsqueeze(-1).expand(-1, -1, 64))
        dm = route.video_dynamic_map.view(1, 2, 16, 32)
        out_perm = dynamic_block_sparse_fwd_torch(
            q_perm.view(1, 2, 256, 64), route.k_permuted, route.v_permuted, dm,
            route.q_cluster_sizes.view(1, 2, 16), route.k_cluster_sizes.view(1, 2, 32))
        base = apply_inverse_permutation(out_perm, q_order.view(1, 2, 256), dim=2)
        repaired, info = core.repair(base, q, k, v, route)
        state = core.repair_state_current
        torch.save({
            "q": q, "k": k, "v": v, "mode": mode,
            "config": {"num_q_centroids": 16, "num_k_centroids": 32, "target_density": 0.25,
                       "kmeans_iter_init": 8, "probe_rows": 16, "repair_rank": 16,
                       "svg_ear_top_p": 0.25, "tol": 1e-4, "seed_k": seeds["k"], "seed_q": seeds["q"]},
            "q_labels": route.q_labels.clone(), "k_labels": route.k_labels.clone(),
            "q_sizes": route.q_cluster_sizes.clone(), "k_sizes": route.k_cluster_sizes.clone(),
            "mask": route.video_dynamic_map.clone(), "q_features": route.q_role_features.clone(),
            "q_iters": route.q_kmeans_iters, "k_iters": route.k_kmeans_iters,
            "base": base.clone(), "repaired": repaired.clone(),
            "probe_rows": route.probe_rows.clone(), "probe_weights": route.probe_weights.clone(),
            "state": tuple(t.clone() for t in state),
            "base_density": route.base_video_density,
        }, os.path.join(HERE, f"config0_{mode}.pt"))
        print(mode, "k_iters", route.k_kmeans_iters, "q_iters", route.q_kmeans_iters,
              "density", info["effective_video_density"])

    q, k, v = synthetic_qkv(4, 64, (4, 8, 8), dtype=torch.float32, seeds=(3, 4, 5))
    calls["n"] = 0
    cfg = n8.N8V6Config(
        num_q_centroids=16, num_k_centroids=32, target_density=0.25,
        kmeans_iter_init=8, kmeans_iter_step=2, probe_rows=16, repair_rank=16,
        selector_policy="attention_mass", selector_budget_mode="fixed_density",
        compile_role_kv_projection=False,
    )
    core = n8.N8V6Core(cfg)
    route = core.route(q, k, v, gqa_group_size=2, total_key_tokens=q.shape[2])
    torch.save({
        "q": q, "k": k, "v": v, "gqa_group_size": 2,
        "config": {"num_q_centroids": 16, "num_k_centroids": 32, "target_density": 0.25,
                   "kmeans_iter_init": 8, "probe_rows": 16, "tol": 1e-4, "seed_k": seeds["k"]},
        "q_labels": route.q_labels.clone(), "k_labels": route.k_labels.clone(),
        "q_sizes": route.q_cluster_sizes.clone(), "k_sizes": route.k_cluster_sizes.clone(),
        "k_centroids": core.k_centroids.clone(), "v_centroids": core.v_centroids.clone(),
        "q_centroids": core.q_centroids.clone(), "mask": route.video_dynamic_map.clone(),
        "q_features": route.q_role_features.clone(), "k_permuted": route.k_permuted.clone(),
        "q_iters": route.q_kmeans_iters, "k_iters": route.k_kmeans_iters,
    }, os.path.join(HERE, "config0_gqa.pt"))
    print("gqa", "k_iters", route.k_kmeans_iters, "q_iters", route.q_kmeans_iters)

    q, k, v = synthetic_qkv(2, 128, (4, 8, 8), dtype=torch.float32, seeds=(6, 7, 8))
    calls["n"] = 0
    cfg = n8.N8V6Config(
        num_q_centroids=16, num_k_centroids=32, target_density=0.25,
        kmeans_iter_init=8, kmeans_iter_step=2, probe_rows=16, repair_rank=16,
        selector_policy="svg_ear_value", selector_budget_mode="fixed_density",
        compile_role_kv_projection=False,
    )
    core = n8.N8V6Core(cfg)
    route = core.route(q, k, v, total_key_tokens=q.shape[2])
    torch.save({
        "q": q, "k": k, "v": v,
        "config": {"num_q_centroids": 16, "num_k_centroids": 32, "target_density": 0.25,
                   "kmeans_iter_init": 8, "probe_rows": 16, "tol": 1e-4, "seed_k": seeds["k"]},
        "q_labels": route.q_labels.clone(), "k_labels": route.k_labels.clone(),
        "q_sizes": route.q_cluster_sizes.clone(), "k_sizes": route.k_cluster_sizes.clone(),
        "mask": route.video_dynamic_map.clone(),
        "q_iters": route.q_kmeans_iters, "k_iters": route.k_kmeans_iters,
    }, os.path.join(HERE, "config0_svg_value.pt"))
    print("svg_value", "k_iters", route.k_kmeans_iters, "q_iters", route.q_kmeans_iters)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py /path/to/SparsePR")
    main(sys.argv[1])
