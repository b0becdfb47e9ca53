"""Route reuse across denoising steps and CFG branches (the Cosmos2.5
adapter's route cache, ``cosmos_predict2.py:840-868, 1193-1400``)."""

import types

import pytest
import torch

import oracle
from sparsepr_b200.route_cache import RouteCache, RouteReuseConfig, _Entry, route_action


def _schedule(cfg, steps, branches):
    """Actions for ``steps`` x ``branches`` calls of one module."""
    entry, out = None, []
    for step in range(steps):
        for _branch in range(branches):
            act = route_action(entry, step=step, config=cfg)
            if act == "refresh":
                entry = _Entry(origin_step=step, last_step=step, route=None)
            entry.last_step = step
            out.append(act)
    return out


def test_route_action_schedule():
    cfg = RouteReuseConfig(dense_first_steps=2, route_refresh_every=4, share_cfg_route=True)
    acts = _schedule(cfg, 8, 2)
    # Steps 0-1 (before the sparse steps) and step 2 (sparse step 0) refresh;
    # the second CFG branch of a step always reuses its first branch's route.
    assert acts[0::2] == ["refresh", "refresh", "refresh", "temporal_reuse", "temporal_reuse",
                          "temporal_reuse", "refresh", "temporal_reuse"]
    assert acts[1::2] == ["cfg_reuse"] * 8
    no_share = RouteReuseConfig(dense_first_steps=0, route_refresh_every=2, share_cfg_route=False)
    assert _schedule(no_share, 4, 1) == ["refresh", "temporal_reuse", "refresh", "temporal_reuse"]
    cache = RouteCache(no_share)
    assert cache.key("m", 1) == ("m", 1) and RouteCache(cfg).key("m", 1) == ("m", 0)
    with pytest.raises(ValueError):
        RouteCache(RouteReuseConfig(route_refresh_every=0))


@pytest.mark.gpu
def test_reused_route_attention_matches_oracle():
    """A reused route attends the CURRENT step's Q/K/V over the cached map."""
    from sparsepr_b200.n8_v6 import N8V6Config, N8V6Core
    from sparsepr_b200.synthetic import synthetic_qkv

    dev = torch.device("cuda:0")
    cfg = N8V6Config(num_q_centroids=32, num_k_centroids=48, target_density=0.3, kmeans_iter_init=6,
                     probe_rows=32, repair_rank=16, role_kv_matmul_precision="highest", kmeans_precision="fp32")
    core = N8V6Core(cfg)
    cache = RouteCache(RouteReuseConfig(dense_first_steps=0, route_refresh_every=2))
    q, k, v = synthetic_qkv(2, 128, (4, 8, 16), dtype=torch.bfloat16)
    q2, k2, v2 = synthetic_qkv(2, 128, (4, 8, 16), dtype=torch.bfloat16, seeds=(7, 8, 9))
    out0, _, i0 = cache.attention(q.to(dev), k.to(dev), v.to(dev), core, module_id=0, step=0, branch=0)
    out1, _, i1 = cache.attention(q.to(dev), k.to(dev), v.to(dev), core, module_id=0, step=0, branch=1)
    _, _, i2 = cache.attention(q2.to(dev), k2.to(dev), v2.to(dev), core, module_id=0, step=1, branch=0)
    _, _, i3 = cache.attention(q2.to(dev), k2.to(dev), v2.to(dev), core, module_id=0, step=2, branch=0)
    assert [i["route_action"] for i in (i0, i1, i2, i3)] == ["refresh", "cfg_reuse", "temporal_reuse", "refresh"]
    assert cache.counts == {"route_refresh_calls": 2, "route_reuse_calls": 2, "cfg_route_reuse_calls": 1,
                            "temporal_route_reuse_calls": 1}
    # Same inputs through the cached route: same attention output, same repair.
    assert torch.equal(i1["base"], i0["base"])
    assert torch.equal(out1, out0)
    # New inputs through the step-0 route: the oracle's attention on the cached map.
    r = i0["route"]
    ql, kl = r.q_labels.cpu().long(), r.k_labels.cpu().long()
    qs, ks = r.q_cluster_sizes.cpu().long(), r.k_cluster_sizes.cpu().long()
    qo, ko = oracle.stable_label_order(ql), oracle.stable_label_order(kl)
    q3, k3, v3 = (t.view(2, -1, 128) for t in (q2, k2, v2))
    ref = oracle.block_sparse_attention(oracle.permute_rows(q3, qo), oracle.permute_rows(k3, ko),
                                        oracle.permute_rows(v3, ko), r.video_dynamic_map.cpu(), qs, ks)
    ref = oracle.inverse_permute_rows(ref, qo)
    got = i2["base"].cpu().view(2, -1, 128)
    torch.testing.assert_close(got.float(), ref.float(), atol=2e-2, rtol=2e-2)
    assert torch.equal(i2["route"].k_sorted_indices, r.k_sorted_indices)


@pytest.mark.gpu
def test_dense_first_steps_run_dense_and_leave_cache():
    """Steps before dense_first_steps are exact dense attention and do not touch
    the cache (cosmos_predict2.py:1509-1520); the first sparse step refreshes."""
    from sparsepr_b200.n8_v6 import N8V6Config, N8V6Core
    from sparsepr_b200.synthetic import synthetic_qkv

    dev = torch.device("cuda:0")
    cfg = N8V6Config(num_q_centroids=16, num_k_centroids=24, target_density=0.3, kmeans_iter_init=4,
                     probe_rows=16, repair_rank=16, role_kv_matmul_precision="highest", kmeans_precision="fp32")
    core = N8V6Core(cfg)
    cache = RouteCache(RouteReuseConfig(dense_first_steps=2, route_refresh_every=4))
    q, k, v = synthetic_qkv(2, 128, (4, 8, 8), dtype=torch.bfloat16)
    assert cache.action(0, step=0) == "dense"
    out, density, info = cache.attention(q.to(dev), k.to(dev), v.to(dev), core, module_id=0, step=0)
    assert info["route_action"] == "dense" and density == 1.0 and not cache.entries
    assert not core.initialized
    ref = oracle.dense_attention_rows(q.view(2, -1, 128), k.view(2, -1, 128), v.view(2, -1, 128))
    torch.testing.assert_close(out.cpu().view(2, -1, 128).float(), ref.float(), atol=2e-2, rtol=2e-2)
    _, _, i2 = cache.attention(q.to(dev), k.to(dev), v.to(dev), core, module_id=0, step=2)
    assert i2["route_action"] == "refresh" and cache.counts["dense_calls"] == 1
