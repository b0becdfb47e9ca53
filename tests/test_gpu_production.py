"""Parity at the benchmarked production settings, on 2 of the 40 heads.

Configs 3 (75,600 tokens, 21x45x80) and 2 (32,760 tokens, 21x30x52): D=128,
Cq=200, Ck=1000, 10 Lloyd iterations with TF32 routing distances, keep 30%
(fixed density), 64 probes, rank 16.  The build's route is fed to the CPU
oracle (``oracle.oracle_sparse_attention(route=...)``), so every stage after
clustering is compared on identical clusters:

* selector masks bit-exact given the build's scores, scores within fp32
  rounding of the oracle's scores on the build's centroids;
* base (pre-repair) output and the repaired output within max-abs 2e-2 and
  cosine >= 0.999 per head (bf16);
* the TF32 assignment at this size: labels equal to the exact fp32 argmin
  wherever the best/second-best gap exceeds the TF32 bound.
"""

import types

import pytest
import torch

import oracle
from sparsepr_b200 import N8V6Config, N8V6Core, kernels as K, sparse_attention
from sparsepr_b200.synthetic import synthetic_qkv_heads

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.999
SETTINGS = dict(num_q_centroids=200, num_k_centroids=1000, target_density=0.3, kmeans_iter_init=10,
                probe_rows=64, repair_rank=16, repair_ridge=0.1, selector_policy="attention_mass",
                selector_budget_mode="fixed_density", kmeans_tol=0.0)
GRIDS = {3: (21, 45, 80), 2: (21, 30, 52)}


def _close(name, got, ref):
    got, ref = got.float().cpu(), ref.float().cpu()
    err = (got - ref).abs().max().item()
    assert err <= ATOL, (name, err)
    for h in range(got.shape[0]):
        cos = torch.nn.functional.cosine_similarity(got[h].flatten(), ref[h].flatten(), dim=0).item()
        assert cos >= COS, (name, h, cos)


@pytest.mark.parametrize("config", [3, 2])
def test_production_layer_matches_oracle_on_build_route(cuda, config):
    grid = GRIDS[config]
    cfg = N8V6Config(**SETTINGS)
    q, k, v = synthetic_qkv_heads(0, 2, 128, grid, device=cuda)
    out, density, info = sparse_attention(q, k, v, N8V6Core(cfg), return_base=True)
    torch.cuda.synchronize()
    r = info["route"]
    bh, n = 2, q.shape[2]
    qc, kc, vc = (t.cpu() for t in (q, k, v))
    ro = types.SimpleNamespace(
        q_labels=r.q_labels.cpu().long(), q_sizes=r.q_cluster_sizes.cpu().long(),
        k_sizes=r.k_cluster_sizes.cpu().long(), mask=r.video_dynamic_map.cpu(), q_features=r.q_role_features.cpu(),
        q_order=r.q_sorted_indices.cpu().long(), k_perm=r.k_permuted.view(bh, -1, 128).cpu(),
        v_perm=r.v_permuted.view(bh, -1, 128).cpu())
    # Selector: masks bit-exact given the scores; the scores themselves on the build's centroids.
    ks = ro.k_sizes
    routed = oracle.select_budget(r.scores.cpu(), ks, r.budgets.cpu())
    assert torch.equal(ro.mask, routed[:, 1:, 1:])
    qcent = oracle.original_centroids(qc.view(bh, n, 128), ro.q_labels, ro.q_sizes)
    sc = oracle.attention_mass_scores(qcent, ro.k_perm, ks)
    fin = torch.isfinite(sc)
    assert torch.equal(fin, torch.isfinite(r.scores.cpu()))
    torch.testing.assert_close(r.scores.cpu()[fin], sc[fin], atol=2e-3, rtol=1e-4)
    # Attention and repair on the build's route.
    ocfg = types.SimpleNamespace(role_q_rank=64, role_k_rank=48, metric_sample_tokens=2048, repair_alpha=1.0,
                                 repair_norm_cap=0.0, **SETTINGS)
    _ref, _r, base_ref, _extra = oracle.oracle_sparse_attention(qc, kc, vc, ocfg, route=ro)
    base = info["base"].cpu()
    _close("base", base, base_ref)
    rows = r.probe_rows.cpu().long()
    q3, k3, v3 = (t.view(bh, n, 128) for t in (qc, kc, vc))
    dense = oracle.dense_attention_rows(torch.gather(q3, 1, rows.unsqueeze(2).expand(-1, -1, 128)), k3, v3)
    state = tuple(t.cpu() for t in info["repair_state"])
    ref = oracle.repair_apply(base, state)
    ref.scatter_(1, rows.unsqueeze(2).expand(-1, -1, 128), dense)
    _close("repaired", out.cpu().view(bh, n, 128), ref)
    pair = oracle.kept_pairs(ro.mask, ro.q_sizes, ks) / float(bh * n * n)
    assert 0.2 <= pair <= 0.35, pair
    assert 0.0 < density <= 1.0


def test_production_tf32_assignment_matches_exact_away_from_ties(cuda):
    """The K-role assignment at config-3 size (75,600 x 1,000 x 48, TF32 with the
    folded bias) and the Q role (x 200 x 64) against the exact argmin."""
    g = torch.Generator().manual_seed(5)
    for k, d in ((1000, 48), (200, 64)):
        x = torch.randn(2, 75600, d, generator=g)
        x = x / x.square().mean(-1, keepdim=True).sqrt()
        c = x[:, torch.randint(0, 75600, (k,), generator=g)] + 0.05 * torch.randn(2, k, d, generator=g)
        got = K.kmeans_assign(x.to(cuda), c.to(cuda), precision="tf32").cpu().long()
        assert K.kmeans_error_code(cuda) == 0
        ref = oracle.euclid_assign(x, c)
        gap = oracle.assign_margin(x, c)
        bound = 4e-3 * ((x * x).sum(-1) + (c * c).sum(-1).amax(-1, keepdim=True))
        clear = gap > bound
        assert clear.float().mean() > 0.5
        assert torch.equal(got[clear], ref[clear]), (k, d, (got[clear] != ref[clear]).sum().item())


def test_config1_standalone_kmeans_matches_oracle(cuda):
    """Config 1 shape (75,600 x 128 bf16 points, K = 256, seeded k-means++ init),
    on 2 of the 40 problems, through the standalone flash_kmeans contract
    (centroids rounded to bf16 after every update, bf16 tensor-core distances).
    One iteration: labels equal to the exact fp32 argmin wherever the top-2 gap
    exceeds 1e-5 (|x|^2 + |c|^2).  Ten iterations: >= 99.9% of labels and the
    centroids (to bf16 rounding) equal to the oracle's run."""
    from sparsepr_b200 import batch_kmeans_Euclid
    from sparsepr_b200.synthetic import kmeans_plus_plus, synthetic_kmeans_points

    x = synthetic_kmeans_points(2, 128, (21, 45, 80), 256, device=cuda, seed=0)
    init = kmeans_plus_plus(x, 256, seed=3)
    xc, ic = x.cpu(), init.cpu()
    lab1, _c1, _s1, _i1 = batch_kmeans_Euclid(x, 256, max_iters=1, tol=0.0, init_centroids=init,
                                             round_centroids_to_input=True)
    assert K.kmeans_error_code(cuda) == 0
    ref1 = oracle.euclid_assign(xc, ic)
    gap = oracle.assign_margin(xc, ic)
    bound = 1e-5 * ((xc.float() ** 2).sum(-1) + (ic ** 2).sum(-1).amax(-1, keepdim=True))
    clear = gap > bound
    assert clear.float().mean() > 0.99
    got1 = lab1.cpu().long()
    assert torch.equal(got1[clear], ref1[clear])
    lab, cent, sizes, iters = batch_kmeans_Euclid(x, 256, max_iters=10, tol=0.0, init_centroids=init,
                                                 round_centroids_to_input=True)
    rl, rc, rs, rit = oracle.batch_kmeans_euclid(xc, 256, 10, 0.0, ic, centroid_dtype=torch.bfloat16)
    assert int(iters.item()) == rit == 10
    gl = lab.cpu().long()
    agree = (gl == rl).float().mean().item()
    assert agree >= 0.999, agree
    # Centroids of the clusters whose members agree in both runs.
    bad = torch.zeros(2, 256, dtype=torch.bool)
    diff = gl != rl
    for b in range(2):
        bad[b, gl[b][diff[b]]] = True
        bad[b, rl[b][diff[b]]] = True
    assert (~bad).float().mean() > 0.9
    torch.testing.assert_close(cent.cpu()[~bad], rc[~bad], atol=2e-2, rtol=1e-2)
