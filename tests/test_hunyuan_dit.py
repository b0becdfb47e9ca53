"""The random-init HunyuanVideo-architecture DiT around the Hunyuan SparsePR boundary.

CPU: the sequence-parallel forward (Ulysses exchange of the video tokens, text
replicated, text output heads all-gathered) on two gloo ranks equals the
one-rank forward, with a dense stand-in for the attention.  GPU: SparsePR
inside the DiT with every key cluster kept matches dense attention under the
boundary's text rules, block by block."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from sparsepr_b200.hunyuan_dit import HunyuanDiT, HunyuanDiTConfig, JointAttention, rope_3d


def dense_joint(q, k, v, n_video, prompt):
    """softmax attention over [1, h, video + text, D] with the Hunyuan boundary's
    key sets: video and prompt rows see video + prompt keys, padding rows see
    padding keys only (hunyuanvideo.py:195-217)."""
    tokens = q.shape[2]
    keep = n_video + prompt
    rows = torch.arange(tokens, device=q.device)
    cols = torch.arange(tokens, device=q.device)
    allowed = torch.where((rows < keep)[:, None], (cols < keep)[None, :], (cols >= keep)[None, :])
    s = q.float() @ k.float().transpose(-1, -2) / q.shape[-1] ** 0.5
    s = s.masked_fill(~allowed, float("-inf"))
    return (torch.softmax(s, dim=-1) @ v.float()).to(q.dtype)


def _tiny(head_dim=16, heads=4):
    axes = (4, 6, 6) if head_dim == 16 else (16, 56, 56)
    return HunyuanDiTConfig(hidden=heads * head_dim, heads=heads, head_dim=head_dim, double_blocks=1,
                            single_blocks=1, text_dim=32, vec_dim=24, rope_axes=axes)


def _inputs(latent_shape, text_tokens, text_dim, vec_dim, device):
    g = torch.Generator().manual_seed(11)
    latent = torch.randn(*latent_shape, generator=g).to(device)
    text = torch.randn(text_tokens, text_dim, generator=g).to(device)
    pooled = torch.randn(vec_dim, generator=g).to(device)
    return latent, text, torch.tensor(500.0, device=device), pooled, torch.tensor(6.0, device=device)


def test_rope_3d_positions():
    cos, sin = rope_3d((2, 3, 4), torch.arange(24), (4, 6, 6), 256.0, "cpu")
    assert cos.shape == (24, 8)
    # Token 0 sits at the origin: no rotation.  Token 5 = (t0, h1, w1): the
    # t channels stay, the h and w channels turn.
    assert torch.allclose(cos[0], torch.ones(8)) and torch.allclose(sin[0], torch.zeros(8))
    assert torch.allclose(cos[5, :2], torch.ones(2)) and not torch.allclose(cos[5, 2:], torch.ones(6))


def test_dit_forward_cpu_shapes():
    cfg = _tiny()
    model = HunyuanDiT(cfg, "cpu", dtype=torch.float32, seed=1)
    latent, text, t, pooled, guid = _inputs((16, 2, 4, 8), 6, cfg.text_dim, cfg.vec_dim, "cpu")
    att = JointAttention(lambda i, q, k, v, n: dense_joint(q, k, v, n, 4))
    out = model.forward(latent, text, t, pooled, guid, att)
    assert out.shape == (2 * 2 * 4, 64) and torch.isfinite(out).all()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sp_main(rank, world, port, out):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _tiny()
        model = HunyuanDiT(cfg, "cpu", dtype=torch.float32, seed=1)
        inputs = _inputs((16, 2, 4, 8), 6, cfg.text_dim, cfg.vec_dim, "cpu")
        att = JointAttention(lambda i, q, k, v, n: dense_joint(q, k, v, n, 4))
        mine = model.forward(*inputs, att, rank=rank, world=world)
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        if rank == 0:
            out.put(torch.cat(parts))
    finally:
        dist.destroy_process_group()


def test_sequence_parallel_forward_matches_one_rank():
    cfg = _tiny()
    model = HunyuanDiT(cfg, "cpu", dtype=torch.float32, seed=1)
    inputs = _inputs((16, 2, 4, 8), 6, cfg.text_dim, cfg.vec_dim, "cpu")
    ref = model.forward(*inputs, JointAttention(lambda i, q, k, v, n: dense_joint(q, k, v, n, 4)))
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sp_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    torch.testing.assert_close(got, ref, atol=1e-4, rtol=1e-4)


@pytest.mark.gpu
def test_dit_sparsepr_all_clusters_kept_matches_dense():
    """Every key cluster kept (top-p budgets clamped to all tokens): SparsePR in
    each block equals dense attention under the boundary's rules within the
    bf16 tolerance (max-abs 2e-2, cosine >= 0.999), and the step is finite."""
    from sparsepr_b200 import N8V6Config
    from sparsepr_b200.hunyuan_dit import SparsePRBlocks

    dev = torch.device("cuda:0")
    cfg = _tiny(head_dim=128, heads=2)
    model = HunyuanDiT(cfg, dev, seed=2)
    inputs = _inputs((16, 4, 16, 32), 40, cfg.text_dim, cfg.vec_dim, dev)
    sp = N8V6Config(num_q_centroids=32, num_k_centroids=48, kmeans_iter_init=6, probe_rows=32, repair_rank=16,
                    selector_policy="svg_ear_value", selector_budget_mode="svg_ear_top_p",
                    adaptive_budget_min_density=1.0, adaptive_budget_max_density=1.0,
                    role_kv_matmul_precision="highest", kmeans_tol=0.0)
    blocks = SparsePRBlocks(sp, cfg.double_blocks + cfg.single_blocks, prompt_length=30)
    errs = []

    def inner(i, q, k, v, n):
        o = blocks(i, q, k, v, n)
        ref = dense_joint(q, k, v, n, 30).float()
        got = o.float()
        cos = torch.nn.functional.cosine_similarity(got.flatten(2), ref.flatten(2), dim=-1)
        errs.append(((got - ref).abs().max().item(), cos.min().item()))
        return o

    out = model.forward(*inputs, JointAttention(inner))
    torch.cuda.synchronize()
    assert out.shape == (4 * 8 * 16, 64) and torch.isfinite(out.float()).all()
    assert len(errs) == 2
    for err, cos in errs:
        assert err < 2e-2 and cos >= 0.999, errs
