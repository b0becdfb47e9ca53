"""Generate golden warm role factors by running the REFERENCE's
``warm_subspace_metric_factor`` (pure torch) on the CPU.

Run in a container that has the reference checkout (it is never read at test
time):

    python tests/golden/make_warm_factor_golden.py /path/to/SparsePR

Inputs: query-sample metrics (uncentered covariances of smooth-field queries)
for a previous and a current denoising step; the previous factor is the exact
top-r factor of the previous metric (the state after a first refresh).  The
function runs with the N8V6Config defaults (2 power iterations,
each_cholesky_qr2, rayleigh_cholesky, ridges 1e-4 / 1e-5).  Output:
``tests/golden/warm_factor.pt``.
"""

from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import torch
    from sparsepr.models.cosmos3.operator_kmeans import metric_factor, warm_subspace_metric_factor

    g = torch.Generator().manual_seed(5)
    cases = []
    for bh, d, rank in ((3, 128, 48), (2, 128, 64)):
        base = torch.randn(bh, 512, d, generator=g) * torch.linspace(0.2, 2.0, d)
        drift = 0.1 * torch.randn(bh, 512, d, generator=g)
        prev_metric = torch.bmm(base.transpose(1, 2), base) / 512
        cur = base + drift
        metric = torch.bmm(cur.transpose(1, 2), cur) / 512
        previous = metric_factor(prev_metric, rank)
        factor, basis, recovered = warm_subspace_metric_factor(
            metric, previous, rank, power_iters=2, orthogonalization="each_cholesky_qr2",
            ritz_mode="rayleigh_cholesky", rayleigh_ridge=1e-4, cholesky_qr_ridge=1e-5, return_basis=True,
            return_recovery_mask=True)
        cases.append(dict(metric=metric, previous=previous, rank=rank, factor=factor, basis=basis,
                          recovered=recovered))
    torch.save(cases, os.path.join(HERE, "warm_factor.pt"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_warm_factor_golden.py /path/to/SparsePR")
    main(sys.argv[1])
