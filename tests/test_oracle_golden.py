"""The CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py) and the reference's selector known-answer test."""

import os
import types

import pytest
import torch

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _cfg(mode):
    return types.SimpleNamespace(
        num_q_centroids=16, num_k_centroids=32, target_density=0.25, kmeans_iter_init=8, probe_rows=16,
        repair_rank=16, repair_ridge=0.1, repair_alpha=1.0, repair_norm_cap=0.0, role_q_rank=64, role_k_rank=48,
        metric_sample_tokens=2048, selector_budget_mode=mode, svg_ear_top_p=0.25,
        adaptive_budget_min_density=0.0, adaptive_budget_max_density=1.0)


@pytest.fixture(scope="module", params=["fixed_density", "svg_ear_top_p"])
def golden(request):
    g = torch.load(os.path.join(GOLDEN, f"config0_{request.param}.pt"))
    out, route, base, extra = oracle.oracle_sparse_attention(
        g["q"], g["k"], g["v"], _cfg(request.param), init_seed=g["config"]["seed_k"], tol=g["config"]["tol"])
    return g, out, route, base, extra


def test_route_matches_reference(golden):
    g, _out, r, _base, _ = golden
    assert torch.equal(r.k_labels, g["k_labels"].long())
    assert torch.equal(r.q_labels, g["q_labels"].long())
    assert torch.equal(r.k_sizes, g["k_sizes"].long())
    assert torch.equal(r.q_sizes, g["q_sizes"].long())
    assert torch.equal(r.mask, g["mask"])
    assert (r.k_iters, r.q_iters) == (g["k_iters"], g["q_iters"])
    # Eigenvector signs are arbitrary; compare the sign-invariant row Gram.
    a, b = r.q_features[:, :64], g["q_features"].float()[:, :64]
    torch.testing.assert_close(a @ a.transpose(1, 2), b @ b.transpose(1, 2), atol=1e-3, rtol=1e-4)


def test_base_attention_matches_reference(golden):
    g, _out, _r, base, _ = golden
    torch.testing.assert_close(base.reshape(g["base"].shape), g["base"], atol=1e-5, rtol=1e-5)


def test_probe_selection_matches_reference(golden):
    g, _out, _r, _base, (state, rows, weights, dense) = golden
    assert torch.equal(rows, g["probe_rows"].long())
    torch.testing.assert_close(weights, g["probe_weights"], atol=1e-6, rtol=1e-6)


def test_repair_fit_matches_reference(golden):
    """Means/scales exactly; the rank-16-of-16-probes basis is rank deficient at
    config 0, so only its 15 well-conditioned columns are compared (up to sign)."""
    g, _out, _r, _base, (state, *_rest) = golden
    for i in range(3):
        torch.testing.assert_close(state[i], g["state"][i], atol=1e-6, rtol=1e-5)
    b_new, b_ref = state[4][:, :, 1:], g["state"][4][:, :, 1:]
    sign = torch.sign((b_new * b_ref).sum(1, keepdim=True))
    torch.testing.assert_close(b_new * sign, b_ref, atol=1e-4, rtol=1e-3)
    torch.testing.assert_close(state[3][:, :, 1:] * sign, g["state"][3][:, :, 1:], atol=1e-4, rtol=1e-3)


def test_repair_apply_matches_reference(golden):
    g, *_ = golden
    base = g["base"].view(2, 256, 64)
    out = oracle.repair_apply(base, g["state"])
    rows = g["probe_rows"].long()
    gidx = rows.unsqueeze(2).expand(-1, -1, 64)
    q3, k3, v3 = (t.reshape(2, 256, 64) for t in (g["q"], g["k"], g["v"]))
    dense = oracle.dense_attention_rows(torch.gather(q3, 1, gidx), k3, v3)
    out.scatter_(1, gidx, dense)
    torch.testing.assert_close(out.view_as(g["repaired"]), g["repaired"], atol=2e-6, rtol=1e-6)


def test_selector_known_answer():
    """The reference's hand-checked selector example (tests/test_n8_extension.py:79-103)."""
    scores = torch.tensor([[[4.0, 3.0, 2.0, 1.0], [1.0, 4.0, 3.0, 2.0]]])
    sizes = torch.tensor([[2, 3, 5, 1]])
    budgets = torch.tensor([[6, 4]])
    routed = oracle.select_budget(scores, sizes, budgets)
    expected = torch.tensor([[True, True, True, False], [False, True, True, False]])
    assert torch.equal(routed[0, 1:, 1:], expected)
    assert routed[0, 0, 0] and routed[0, 1:, 0].all()
    ids, counts = oracle.compact_selected(expected)
    assert counts.tolist() == [3, 2]
    assert ids[0, :3].tolist() == [0, 1, 2] and ids[1, :2].tolist() == [1, 2]


def test_selector_crossing_rules():
    """GPU-path rule: no crossing cluster once every positive cluster fits,
    none for a zero budget, ties broken toward the lower cluster id."""
    scores = torch.tensor([[[1.0, 1.0, 0.5, float("-inf")]]])
    sizes = torch.tensor([[3, 3, 2, 0]])
    assert oracle.select_budget(scores, sizes, torch.tensor([[100]]))[0, 1, 1:].tolist() == [True, True, True, False]
    assert oracle.select_budget(scores, sizes, torch.tensor([[0]]))[0, 1, 1:].tolist() == [False] * 4
    assert oracle.select_budget(scores, sizes, torch.tensor([[2]]))[0, 1, 1:].tolist() == [True, False, False, False]


def test_kmeans_loop_contract():
    """tol stop keeps the pre-update centroids; labels/sizes from the last assignment."""
    torch.manual_seed(0)
    x = torch.randn(2, 300, 16)
    init = x[:, :8].clone()
    l1, c1, s1, it1 = oracle.batch_kmeans_euclid(x, 8, 50, 1e-6, init)
    assert it1 < 50
    assert torch.equal(l1, oracle.euclid_assign(x, c1))
    assert torch.equal(s1.sum(1), torch.full((2,), 300))


def test_oracle_svg_ear_value_scores_match_reference_kernel():
    """The oracle's value-error scores against the reference Triton kernel's own
    outputs (run on CPU by Triton's interpreter, tests/golden/make_svg_golden.py)."""
    cases = torch.load(os.path.join(os.path.dirname(__file__), "golden", "svg_ear_value_scores.pt"))
    for c in cases:
        got = oracle.svg_ear_value_error_scores(c["q_centroids"], c["k_sorted"], c["v_sorted"], c["k_centroids"],
                                                c["v_centroids"], c["k_sizes"])
        ref = c["scores"]
        fin = torch.isfinite(ref)
        assert torch.equal(fin, torch.isfinite(got))
        assert (~fin).any()  # empty clusters score -inf
        torch.testing.assert_close(got[fin], ref[fin], atol=1e-4, rtol=1e-5)


def test_oracle_warm_factor_matches_reference():
    """The oracle's warm subspace factor against the reference's own
    warm_subspace_metric_factor (tests/golden/make_warm_factor_golden.py)."""
    cases = torch.load(os.path.join(os.path.dirname(__file__), "golden", "warm_factor.pt"))
    for c in cases:
        f, b, rec = oracle.warm_subspace_metric_factor(c["metric"], c["previous"], c["rank"])
        assert torch.equal(rec, c["recovered"])
        torch.testing.assert_close(b, c["basis"], atol=1e-5, rtol=1e-4)
        torch.testing.assert_close(f, c["factor"], atol=1e-5, rtol=1e-4)


def test_gqa_route_matches_reference():
    """GQA route (4 query heads, group 2) against the reference's own route."""
    g = torch.load(os.path.join(GOLDEN, "config0_gqa.pt"))
    cfg = _cfg("fixed_density")
    r = oracle.oracle_route(g["q"], g["k"], g["v"], cfg, init_seed=g["config"]["seed_k"], tol=g["config"]["tol"],
                            gqa_group_size=g["gqa_group_size"])
    assert torch.equal(r.k_labels, g["k_labels"].long())
    assert torch.equal(r.q_labels, g["q_labels"].long())
    assert torch.equal(r.k_sizes, g["k_sizes"].long())
    assert torch.equal(r.q_sizes, g["q_sizes"].long())
    assert torch.equal(r.mask, g["mask"])
    assert (r.k_iters, r.q_iters) == (g["k_iters"], g["q_iters"])
    # K/V centroids stay per native KV head; the route's are per query head.
    torch.testing.assert_close(r.k_centroids[::2], g["k_centroids"].float(), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(r.v_centroids[::2], g["v_centroids"].float(), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(r.q_centroids, g["q_centroids"].float(), atol=1e-5, rtol=1e-5)
    # Each query head permutes its own K rows by the group's labels.  The
    # reference's argsort is not stable, so rows are compared per cluster as
    # sorted sets rather than in order.
    ref_perm = g["k_permuted"].reshape(r.k_perm.shape)
    offs = torch.cat((torch.zeros(4, 1, dtype=torch.long), r.k_sizes.cumsum(1)), 1)
    for h in range(4):
        for c in range(r.k_sizes.shape[1]):
            a, b = int(offs[h, c]), int(offs[h, c + 1])
            mine = r.k_perm[h, a:b]
            ref = ref_perm[h, a:b]
            assert torch.equal(mine[mine[:, 0].argsort()], ref[ref[:, 0].argsort()])
    with pytest.raises(ValueError):
        oracle.oracle_route(g["q"], g["k"], g["v"], cfg, gqa_group_size=3)


def test_svg_value_route_matches_reference():
    """Route with the SVG-EAR value-error selector (the reference's default policy)
    against the reference's own route, its Triton scorer run on the CPU."""
    g = torch.load(os.path.join(GOLDEN, "config0_svg_value.pt"))
    cfg = _cfg("fixed_density")
    cfg.selector_policy = "svg_ear_value"
    r = oracle.oracle_route(g["q"], g["k"], g["v"], cfg, init_seed=g["config"]["seed_k"], tol=g["config"]["tol"])
    assert torch.equal(r.k_labels, g["k_labels"].long())
    assert torch.equal(r.q_labels, g["q_labels"].long())
    assert torch.equal(r.k_sizes, g["k_sizes"].long())
    assert torch.equal(r.q_sizes, g["q_sizes"].long())
    assert (r.k_iters, r.q_iters) == (g["k_iters"], g["q_iters"])
    assert torch.equal(r.mask, g["mask"])


def route_fixture_inputs():
    """The two steps' inputs of tests/golden/make_route_golden.py (regenerated)."""
    import sys

    sys.path.insert(0, GOLDEN)
    try:
        from make_route_golden import CONFIG, inputs
    finally:
        sys.path.remove(GOLDEN)
    return CONFIG, inputs()


def test_two_call_route_matches_reference():
    """Cold then warm route (D = 128): the oracle core against the reference's own
    N8V6Core run twice on the CPU: labels, sizes, map and iteration counts exact,
    centroids to fp32 rounding."""
    fx = torch.load(os.path.join(GOLDEN, "route_d128_two_calls.pt"))
    config, steps = route_fixture_inputs()
    cfg = types.SimpleNamespace(role_q_rank=64, role_k_rank=48, metric_sample_tokens=2048, svg_ear_top_p=0.85,
                                adaptive_budget_min_density=0.0, adaptive_budget_max_density=1.0, **config)
    core = oracle.OracleCore(cfg, init_seed=fx["config"]["seed_k"], tol=fx["config"]["tol"])
    for call, (q, k, v) in zip(fx["calls"], steps):
        assert [float(t.double().sum()) for t in (q, k, v)] == call["input_sums"]
        r = core.route(q, k, v)
        assert torch.equal(r.k_labels, call["k_labels"].long())
        assert torch.equal(r.q_labels, call["q_labels"].long())
        assert torch.equal(r.k_sizes, call["k_sizes"].long())
        assert torch.equal(r.q_sizes, call["q_sizes"].long())
        assert torch.equal(r.mask, call["mask"])
        assert (r.k_iters, r.q_iters) == (call["k_iters"], call["q_iters"])
        for name in ("k_centroids", "v_centroids", "q_centroids"):
            torch.testing.assert_close(getattr(r, name), call[name].float(), atol=1e-5, rtol=1e-5)
