"""The build's route against the reference's own route (D = 128), two calls.

``tests/golden/route_d128_two_calls.pt`` holds the reference ``N8V6Core``'s
cold and warm routes run on the CPU (``make_route_golden.py``).  The build
starts its cold k-means from the same rows (seeds 100 / 101) with fp32
(3xTF32) distances and the reference's ``tol = 1e-4``, then takes a warm
second call (projected previous centroids, warm subspace factors,
``kmeans_iter_step`` iterations).  Role factors come from a different
eigensolver (Jacobi here, LAPACK there), so features agree to fp32 rounding
only; labels may flip on near ties, which the test counts and bounds, and
every iteration count, size and the cluster-pair map must otherwise match.
"""

import os
import sys

import pytest
import torch

from sparsepr_b200 import N8V6Config, N8V6Core
from sparsepr_b200.synthetic import random_init_indices

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _fixture():
    sys.path.insert(0, GOLDEN)
    try:
        from make_route_golden import CONFIG, inputs
    finally:
        sys.path.remove(GOLDEN)
    return CONFIG, inputs(), torch.load(os.path.join(GOLDEN, "route_d128_two_calls.pt"))


def test_two_call_route_matches_reference(cuda):
    config, steps, fx = _fixture()
    cfg = N8V6Config(**config, kmeans_tol=fx["config"]["tol"], kmeans_precision="fp32",
                     role_kv_matmul_precision="highest")
    bh, n = 2, steps[0][0].shape[2]
    init = (random_init_indices(bh, n, cfg.num_k_centroids, fx["config"]["seed_k"]).to(cuda),
            random_init_indices(bh, n, cfg.num_q_centroids, fx["config"]["seed_q"]).to(cuda))
    core = N8V6Core(cfg, init_indices=init)
    report = []
    for i, ((q, k, v), call) in enumerate(zip(steps, fx["calls"])):
        r = core.route(q.to(cuda), k.to(cuda), v.to(cuda))
        kl, ql = r.k_labels.cpu().long(), r.q_labels.cpu().long()
        k_flips = int((kl != call["k_labels"].long()).sum())
        q_flips = int((ql != call["q_labels"].long()).sum())
        mask_diff = int((r.video_dynamic_map.cpu() != call["mask"]).sum())
        k_it = int(r.extras["k_iters_done"].item())
        q_it = int(r.extras["q_iters_done"].item())
        report.append(dict(call=i, k_flips=k_flips, q_flips=q_flips, mask_diff=mask_diff, k_iters=(k_it, call["k_iters"]),
                           q_iters=(q_it, call["q_iters"])))
        assert (k_it, q_it) == (call["k_iters"], call["q_iters"]), report
        # Near-tie flips: at most 0.2% of the points of a call.
        assert k_flips <= 0.002 * bh * n and q_flips <= 0.002 * bh * n, report
        if k_flips == 0 and q_flips == 0:
            assert torch.equal(r.k_cluster_sizes.cpu().long(), call["k_sizes"].long()), report
            assert torch.equal(r.q_cluster_sizes.cpu().long(), call["q_sizes"].long()), report
            assert mask_diff == 0, report
    print(report)
