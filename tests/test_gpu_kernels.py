"""Parity of each CUDA kernel (through the C ABI) against the CPU oracle."""

import pytest
import torch

import oracle
from sparsepr_b200 import kernels as K
from sparsepr_b200.synthetic import synthetic_kmeans_points

pytestmark = pytest.mark.gpu


def _near_tie_free(x, c, rel):
    """Points whose best/second-best gap exceeds a rounding bound of the distance."""
    gap = oracle.assign_margin(x, c)
    scale = (x.double() ** 2).sum(-1) + (c.double() ** 2).sum(-1).max(-1, keepdim=True).values
    return gap > rel * scale


# fp32 (3xTF32) distances: exact labels off fp32 near ties.  tf32 (the
# reference's GPU arithmetic): exact labels where the gap exceeds the TF32
# dot-product error bound (~2^-9 of |x|^2 + |c|^2).
@pytest.mark.parametrize("d,dtype,precision,rel", [
    (48, torch.float32, "fp32", 1e-5), (64, torch.float32, "fp32", 1e-5), (16, torch.float32, "fp32", 1e-5),
    (48, torch.float32, "tf32", 4e-3), (128, torch.bfloat16, "tf32", 4e-3), (96, torch.float32, "tf32", 4e-3),
    (64, torch.bfloat16, "fp32", 1e-5)])
def test_assign_matches_oracle(cuda, d, dtype, precision, rel):
    g = torch.Generator().manual_seed(d)
    x = torch.randn(3, 1537, d, generator=g).to(dtype)
    c = torch.randn(3, 300, d, generator=g)
    ref = oracle.euclid_assign(x, c)
    got = K.kmeans_assign(x.to(cuda), c.to(cuda), precision).cpu().long()
    assert K.kmeans_error_code(cuda) == 0
    ok = _near_tie_free(x, c, rel)
    assert ok.float().mean() > 0.5
    assert torch.equal(got[ok], ref[ok])
    assert (got == ref).float().mean() > 0.98


@pytest.mark.parametrize("precision", ["fp32", "tf32"])
@pytest.mark.parametrize("d", [16, 48, 64])
def test_assign_ties_go_to_lowest_index(cuda, precision, d):
    x = torch.zeros(2, 300, d)
    c = torch.zeros(2, 200, d)  # every centroid at distance 0
    assert K.kmeans_assign(x.to(cuda), c.to(cuda), precision).max().item() == 0


@pytest.mark.parametrize("precision", ["fp32", "tf32"])
def test_assign_coincident_points_clamp_to_zero(cuda, precision):
    """Points equal to a centroid that appears several times: the distance is
    0 up to rounding (clamped at 0 by the reference), so the lowest copy wins."""
    g = torch.Generator().manual_seed(5)
    c = torch.randn(2, 300, 48, generator=g) * 3
    c[:, 150] = c[:, 40]
    c[:, 250] = c[:, 40]
    x = torch.randn(2, 700, 48, generator=g) * 3
    x[:, :100] = c[:, 40:41]
    x[:, 100:200] = c[:, 5:6]
    got = K.kmeans_assign(x.to(cuda), c.to(cuda), precision).cpu()
    assert (got[:, :100] == 40).all()
    assert (got[:, 100:200] == 5).all()
    assert torch.equal(got.long(), oracle.euclid_assign(x, c)) or (got.long() == oracle.euclid_assign(x, c)).float().mean() > 0.99


@pytest.mark.parametrize("n,k", [(1, 1), (5000, 7), (70001, 1000), (4097, 3000)])
def test_label_sort_is_stable_counting_sort(cuda, n, k):
    g = torch.Generator().manual_seed(n)
    labels = torch.randint(0, k, (2, n), generator=g, dtype=torch.int32)
    labels[1, : n // 2] = 0  # skewed cluster sizes
    sizes, offsets, order = K.label_sort(labels.to(cuda), k)
    ref_sizes = torch.zeros(2, k, dtype=torch.long).scatter_add_(1, labels.long(), torch.ones(2, n, dtype=torch.long))
    assert torch.equal(order.cpu().long(), oracle.stable_label_order(labels))
    assert torch.equal(sizes.cpu().long(), ref_sizes)
    assert torch.equal(offsets.cpu().long(), oracle.cluster_offsets(ref_sizes))


@pytest.mark.parametrize("dtype,d", [(torch.bfloat16, 128), (torch.float32, 48), (torch.float32, 64)])
def test_centroid_means_and_permute(cuda, dtype, d):
    g = torch.Generator().manual_seed(7)
    n, k = 3001, 50
    x = torch.randn(2, n, d, generator=g).to(dtype)
    labels = torch.randint(0, k - 5, (2, n), generator=g, dtype=torch.int32)  # last 5 clusters empty
    fallback = torch.randn(2, k, d, generator=g)
    sizes, offsets, order = K.label_sort(labels.to(cuda), k)
    means, xp = K.centroid_means(x.to(cuda), order, offsets, k, fallback.to(cuda), permute=True)
    ref = oracle.original_centroids(x, labels, sizes.cpu().long(), fallback)
    torch.testing.assert_close(means.cpu(), ref, atol=1e-5, rtol=1e-5)
    assert torch.equal(xp.cpu(), oracle.permute_rows(x, oracle.stable_label_order(labels)))


def test_permute_inverse_round_trip(cuda):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, 999, 128, generator=g).to(torch.bfloat16).to(cuda)
    idx = torch.stack([torch.randperm(999, generator=g) for _ in range(3)]).to(torch.int32).to(cuda)
    y = K.permute_rows(x, idx)
    assert torch.equal(y.cpu(), oracle.permute_rows(x.cpu(), idx.cpu()))
    assert torch.equal(K.permute_rows(y, idx, inverse=True), x)


def test_kmeans_lloyd_matches_oracle(cuda):
    x = synthetic_kmeans_points(2, 64, (4, 12, 16), 24, dtype=torch.float32, seed=5)
    init = x[:, torch.randperm(x.shape[1], generator=torch.Generator().manual_seed(1))[:24]].clone()
    lr, cr, sr, itr = oracle.batch_kmeans_euclid(x, 24, 6, 0.0, init)
    l, c, s, off, order, it = K.kmeans_lloyd(x.to(cuda), init.to(cuda), 6, 0.0, precision="fp32")
    assert it.item() == itr == 6
    assert (l.cpu().long() == lr).float().mean() > 0.999
    if torch.equal(l.cpu().long(), lr):
        torch.testing.assert_close(c.cpu(), cr, atol=1e-4, rtol=1e-4)
        assert torch.equal(s.cpu().long(), sr)
        assert torch.equal(order.cpu().long(), oracle.stable_label_order(lr))


def test_kmeans_tol_stops_on_device(cuda):
    x = synthetic_kmeans_points(1, 32, (2, 8, 8), 8, dtype=torch.float32, seed=2)
    init = x[:, :8].clone()
    _l, _c, _s, itr = oracle.batch_kmeans_euclid(x, 8, 40, 1e-3, init)
    _l2, _c2, _s2, _off, _order, it = K.kmeans_lloyd(x.to(cuda), init.to(cuda), 40, 1e-3, precision="fp32")
    assert it.item() == itr < 40


def test_kmeans_bf16_rounded_centroids(cuda):
    x = synthetic_kmeans_points(2, 128, (3, 10, 12), 16, dtype=torch.bfloat16, seed=4)
    init = x[:, :16].float().clone()
    lr, _cr, _sr, _ = oracle.batch_kmeans_euclid(x, 16, 4, 0.0, init, centroid_dtype=torch.bfloat16)
    l, c, *_ = K.kmeans_lloyd(x.to(cuda), init.to(cuda), 4, 0.0, round_centroids_to_input=True)
    assert (l.cpu().long() == lr).float().mean() > 0.999
    assert torch.equal(c.cpu().to(torch.bfloat16).float(), c.cpu())


@pytest.mark.parametrize("bh,n,cq,ck,used,qscale", [
    (2, 1200, 40, 33, 30, 1.0),      # a few empty clusters at the end
    (3, 5000, 200, 250, 250, 3.0),   # two centroid tiles, chunk and tile boundaries inside clusters
    (1, 3000, 20, 5, 5, 1.0),        # clusters much longer than a 128-token tile
    (2, 700, 129, 64, 20, 2.0),      # most clusters empty; one row in the second centroid tile
])
def test_attention_mass_scores(cuda, bh, n, cq, ck, used, qscale):
    g = torch.Generator().manual_seed(11 + n)
    k = torch.randn(bh, n, 128, generator=g).to(torch.bfloat16)
    lab = torch.randint(0, used, (bh, n), generator=g)
    sizes = torch.zeros(bh, ck, dtype=torch.long).scatter_add_(1, lab, torch.ones_like(lab))
    qc = torch.randn(bh, cq, 128, generator=g) * qscale
    ref = oracle.attention_mass_scores(qc, k, sizes)
    off = oracle.cluster_offsets(sizes).to(torch.int32).to(cuda)
    got = K.attention_mass_scores(qc.to(cuda), k.to(cuda), off).cpu()
    assert K.scores_error_code() == 0
    fin = torch.isfinite(ref)
    assert torch.equal(fin, torch.isfinite(got))
    torch.testing.assert_close(got[fin], ref[fin], atol=2e-4, rtol=1e-5)


def test_svg_ear_value_scores(cuda):
    """Value-error scores against the oracle: on the fixture inputs pinned to the
    reference kernel, and on a larger case with chunk and tile boundaries."""
    import os

    cases = torch.load(os.path.join(os.path.dirname(__file__), "golden", "svg_ear_value_scores.pt"))
    g = torch.Generator().manual_seed(21)
    bh, n, cq, ck = 2, 5000, 200, 300
    lab = torch.randint(0, ck - 5, (bh, n), generator=g)
    sizes = torch.zeros(bh, ck, dtype=torch.long).scatter_add_(1, lab, torch.ones_like(lab)).int()
    cases.append(dict(q_centroids=torch.randn(bh, cq, 128, generator=g), k_sorted=torch.randn(bh, n, 128, generator=g).bfloat16(),
                      v_sorted=torch.randn(bh, n, 128, generator=g).bfloat16(), k_centroids=torch.randn(bh, ck, 128, generator=g),
                      v_centroids=torch.randn(bh, ck, 128, generator=g), k_sizes=sizes))
    for c in cases:
        ref = oracle.svg_ear_value_error_scores(c["q_centroids"], c["k_sorted"], c["v_sorted"], c["k_centroids"],
                                                c["v_centroids"], c["k_sizes"])
        off = oracle.cluster_offsets(c["k_sizes"].long()).to(torch.int32).to(cuda)
        got = K.svg_ear_value_scores(c["q_centroids"].to(cuda), c["k_sorted"].to(cuda), c["v_sorted"].to(cuda),
                                     c["k_centroids"].to(cuda), c["v_centroids"].to(cuda), off).cpu()
        assert K.scores_error_code() == 0
        fin = torch.isfinite(ref)
        assert torch.equal(fin, torch.isfinite(got))
        torch.testing.assert_close(got[fin], ref[fin], atol=2e-3, rtol=0)


def test_warm_role_factor_matches_oracle(cuda):
    """Warm subspace factor update (Cholesky-QR and ridge-Cholesky kernels) on the
    inputs pinned to the reference, against the oracle."""
    import os

    from sparsepr_b200.n8_v6 import warm_subspace_metric_factor

    cases = torch.load(os.path.join(os.path.dirname(__file__), "golden", "warm_factor.pt"))
    for c in cases:
        f, b, rec = warm_subspace_metric_factor(c["metric"].to(cuda), c["previous"].to(cuda), c["rank"])
        fo, bo, reco = oracle.warm_subspace_metric_factor(c["metric"], c["previous"], c["rank"])
        assert torch.equal(rec.cpu(), reco)
        torch.testing.assert_close(b.cpu(), bo, atol=2e-4, rtol=1e-3)
        torch.testing.assert_close(f.cpu(), fo, atol=2e-4, rtol=1e-3)


def test_cholesky_kernels_report_failure(cuda):
    bad = -torch.eye(8).expand(2, 8, 8).clone()  # negative definite: every attempt fails
    l, failed = K.ridge_cholesky(bad.to(cuda), torch.ones(2, device=cuda), 1e-4)
    assert failed.all() and torch.equal(l.cpu(), torch.eye(8).expand(2, 8, 8))
    x = torch.randn(2, 16, 4)
    x[1, :, 1] = x[1, :, 0]  # rank deficient: Cholesky-QR of the second problem fails
    out, failed = K.cholesky_qr(x.to(cuda), 1e-12)
    assert failed.tolist() == [False, True]
    q = out[0].cpu()
    torch.testing.assert_close(q.T @ q, torch.eye(4), atol=1e-4, rtol=0)


def test_selector_known_answer(cuda):
    """tests/test_n8_extension.py:79-103 of the reference, through the C ABI."""
    scores = torch.tensor([[[4.0, 3.0, 2.0, 1.0], [1.0, 4.0, 3.0, 2.0]]], device=cuda)
    sizes = torch.tensor([[2, 3, 5, 1]], device=cuda, dtype=torch.int32)
    budgets = torch.tensor([[6, 4]], device=cuda, dtype=torch.int32)
    routed, ids, counts = K.select_budget(scores, sizes, budgets)
    expected = torch.tensor([[True, True, True, False], [False, True, True, False]], device=cuda)
    assert torch.equal(routed[0, 1:, 1:], expected)
    assert routed[0, 0, 0].item() and routed[0, 1:, 0].all().item()
    assert not routed[0, 0, 1:].any().item()
    assert counts.tolist() == [[3, 2]]
    assert ids[0, 0, :3].tolist() == [0, 1, 2] and ids[0, 1, :2].tolist() == [1, 2]


@pytest.mark.parametrize("ck", [1, 37, 1000, 2048])
def test_selector_matches_oracle_bit_exact(cuda, ck):
    g = torch.Generator().manual_seed(ck)
    bh, cq = 3, 17
    scores = torch.randn(bh, cq, ck, generator=g)
    scores[:, :, ::7] = scores[:, :, :1].clone()  # ties
    sizes = torch.randint(0, 50, (bh, ck), generator=g)
    scores = torch.where(sizes.unsqueeze(1) > 0, scores, torch.full_like(scores, float("-inf")))
    budgets = torch.randint(0, int(sizes.sum(1).max()) + 10, (bh, cq), generator=g)
    budgets[0, 0] = 0
    ref = oracle.select_budget(scores, sizes, budgets)
    routed, ids, counts = K.select_budget(scores.to(cuda), sizes.to(torch.int32).to(cuda),
                                          budgets.to(torch.int32).to(cuda))
    assert torch.equal(routed.cpu(), ref)
    rid, rcnt = oracle.compact_selected(ref[:, 1:, 1:])
    assert torch.equal(counts.cpu(), rcnt)
    assert torch.equal(ids.cpu(), rid)


@pytest.mark.parametrize("n", [64, 128, 48, 2])
def test_sym_eig_matches_lapack(cuda, n):
    g = torch.Generator().manual_seed(n)
    x = torch.randn(5, 3 * n + 7, n, generator=g)
    a = x.transpose(1, 2) @ x / x.shape[1]
    a[1] = a[1] * 0  # all-zero matrix
    a[2, :, :] = torch.diag(torch.arange(n, 0, -1).float())  # already diagonal, descending
    w, v = K.sym_eig(a.to(cuda))
    w, v = w.cpu().double(), v.cpu().double()
    wr = torch.linalg.eigvalsh(a.double())
    scale = wr.abs().amax(dim=1, keepdim=True).clamp_min(1.0)
    # fp32 Jacobi: eigenvalues to ~1e-5 of the spectral radius (LAPACK fp64 as truth)
    assert ((w - wr).abs() / scale).max().item() < 2e-4
    ad = a.double()
    resid = (ad @ v - v * w.unsqueeze(1)).abs().amax(dim=(1, 2)) / scale.squeeze(1)
    assert resid.max().item() < 1e-4
    eye = torch.eye(n, dtype=torch.float64)
    assert (v.transpose(1, 2) @ v - eye).abs().max().item() < 1e-4
    assert torch.all(w[:, 1:] >= w[:, :-1])


@pytest.mark.parametrize("n,top", [(128, 64), (128, 48), (64, 16), (64, 64)])
def test_sym_eig_top_matches_lapack(cuda, n, top):
    """Top-``top`` eigenpairs only: all eigenvalues as the full call returns
    them, the last ``top`` columns hold orthonormal eigenvectors (residual
    and orthogonality as in the full test), the other columns are zero; the
    zero matrix (handed to the Jacobi fallback) still yields valid pairs."""
    g = torch.Generator().manual_seed(n + top)
    x = torch.randn(4, 3 * n + 7, n, generator=g)
    a = x.transpose(1, 2) @ x / x.shape[1]
    a[1] = a[1] * 0
    w_full, _ = K.sym_eig(a.to(cuda))
    w, v = K.sym_eig(a.to(cuda), top=top)
    assert torch.equal(w.cpu(), w_full.cpu())
    w, v = w.cpu().double(), v.cpu().double()
    wr = torch.linalg.eigvalsh(a.double())
    scale = wr.abs().amax(dim=1, keepdim=True).clamp_min(1.0)
    assert ((w - wr).abs() / scale).max().item() < 2e-4
    vt, wt = v[:, :, n - top:], w[:, n - top:]
    resid = (a.double() @ vt - vt * wt.unsqueeze(1)).abs().amax(dim=(1, 2)) / scale.squeeze(1)
    assert resid.max().item() < 1e-4
    eye = torch.eye(top, dtype=torch.float64)
    assert (vt.transpose(1, 2) @ vt - eye).abs().max().item() < 1e-4
    if top < n:
        zero_cols = v[[0, 2, 3], :, : n - top]  # matrix 1 went through the full fallback
        assert torch.count_nonzero(zero_cols).item() == 0
    with pytest.raises(RuntimeError):
        K.sym_eig(a.to(cuda), top=n + 1)


@pytest.mark.parametrize("precision", ["tf32", "fp32"])
def test_assign_many_items_per_cta(cuda, precision):
    """Persistent assignment with many point tiles per CTA and 8 centroid tiles
    (the config-3 K-role shape class) completes, reports no device error and
    agrees with the oracle away from near ties."""
    g = torch.Generator().manual_seed(17)
    x = torch.randn(4, 20000, 48, generator=g)
    c = torch.randn(4, 1000, 48, generator=g)
    got = K.kmeans_assign(x.to(cuda), c.to(cuda), precision)
    assert K.kmeans_error_code(cuda) == 0
    ref = oracle.euclid_assign(x, c)
    rel = 1e-5 if precision == "fp32" else 4e-3
    ok = _near_tie_free(x, c, rel)
    assert torch.equal(got.cpu().long()[ok], ref[ok])


@pytest.mark.parametrize("m,r", [(64, 128), (16, 64), (128, 3)])
def test_chol_solve_matches_lapack(cuda, m, r):
    g = torch.Generator().manual_seed(m)
    x = torch.randn(3, m, 2 * m, generator=g)
    a = x @ x.transpose(1, 2) / (2 * m) + 0.1 * torch.eye(m)
    b = torch.randn(3, m, r, generator=g)
    ref = torch.linalg.solve(a.double(), b.double())
    got = K.chol_solve(a.to(cuda), b.to(cuda)).cpu().double()
    assert ((got - ref).abs().max() / ref.abs().max()).item() < 1e-4
    bad = -torch.eye(m).expand(1, m, m)  # not positive definite: non-finite, no error
    assert not torch.isfinite(K.chol_solve(bad.to(cuda), b[:1].to(cuda))).all()


@pytest.mark.parametrize("r", [48, 64, 16])
def test_role_projection_matches_fp64(cuda, r):
    """Tensor-core role projection (bf16 tokens x 3-part bf16 split of the fp32
    factor) against fp64: K role (one RMS per problem) and Q role (per-row RMS),
    with a ragged last tile."""
    g = torch.Generator().manual_seed(r)
    x = torch.randn(3, 1000, 128, generator=g).bfloat16()
    f = torch.randn(3, 128, r, generator=g) * 0.3
    raw = torch.bmm(x.double(), f.double())
    k_ref = raw / raw.square().mean(dim=(1, 2), keepdim=True).sqrt()
    q_ref = raw / raw.square().mean(dim=2, keepdim=True).sqrt()
    kf, ks = K.role_projection(x.to(cuda), f.to(cuda), "global")
    qf, none = K.role_projection(x.to(cuda), f.to(cuda), "row")
    assert K.role_projection_error_code() == 0 and none is None
    torch.testing.assert_close(kf.cpu().double(), k_ref, atol=2e-6, rtol=2e-5)
    torch.testing.assert_close(qf.cpu().double(), q_ref, atol=2e-6, rtol=2e-5)
    torch.testing.assert_close(ks.cpu().view(-1).double(), raw.square().mean(dim=(1, 2)).sqrt(), rtol=1e-5, atol=0)


def test_probe_representatives_match_oracle(cuda):
    """Role-equal probes through the sorted-order kernel against the oracle's
    scatter formulation; two identical rows nearest to their cluster mean go
    to the lower token."""
    from sparsepr_b200.n8_v6 import select_role_equal_probes

    g = torch.Generator().manual_seed(8)
    bh, n, r, k = 3, 3000, 64, 40
    feats = torch.randn(bh, n, r, generator=g)
    labels = torch.randint(0, k - 3, (bh, n), generator=g)  # three empty clusters
    # Cluster 5 = tokens {10, 20, 21, 2000}: 10 and 2000 equal p, 20 and 21 at p +- 5.
    labels[labels == 5] = 6
    labels[:, [10, 20, 21, 2000]] = 5
    p = feats[:, 10].clone()
    feats[:, 2000] = p
    feats[:, 20] = p + 5
    feats[:, 21] = p - 5
    order = oracle.stable_label_order(labels).to(torch.int32)
    sizes = torch.zeros(bh, k, dtype=torch.long).scatter_add_(1, labels, torch.ones_like(labels))
    offsets = torch.cat((torch.zeros(bh, 1, dtype=torch.long), sizes.cumsum(1)), 1).to(torch.int32)
    best = K.probe_representatives(feats.to(cuda), order.to(cuda), offsets.to(cuda)).cpu().long()
    assert (best[:, k - 3:] == n).all()
    assert (best[:, 5] == 10).all()
    rows, w = select_role_equal_probes(feats.to(cuda), labels.to(cuda), k, 32, order=order.to(cuda),
                                       offsets=offsets.to(cuda))
    rows_ref, w_ref = oracle.select_role_equal_probes(feats, labels, k, 32)
    assert (rows.cpu() == rows_ref).float().mean().item() >= 0.99
    torch.testing.assert_close(w.cpu(), w_ref.float(), atol=1e-5, rtol=1e-5)
