"""Benchmark: one SparsePR attention layer at the Wan2.2-720p shape (config 3).

Step = one cold ``sparse_attention`` call on 75,600 tokens x 40 heads x 128
(bf16): role factors, K and Q Lloyd k-means (10 iterations each), centroid
means + permutes, attention-mass scores, budgeted selection (keep 30% of
key tokens per query cluster), block-sparse attention, 64 dense probe rows,
rank-16 repair.  Heads are sharded across ranks (``--gpus N`` under torchrun);
no collective runs on the data path.

Metric: kept TFLOP/s = 4*D*(selected_pairs + probe_pairs) / layer time, the
reference's FLOP audit (``src/sparsepr/adapters/wan22.py:183-190``), summed
over ranks; ``ms_per_step`` is the layer latency (max over ranks).

``--impl reference`` times the reference algorithm's CPU implementation (the
oracle restatement under ``oracle/``; the reference itself is Python and does
not travel to the GPU box) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "SparsePR attn layer ms + kept-TFLOPS at 75.6K tok/40 heads, 1/2/4/8 B200"
CONFIGS = {
    3: dict(grid=(21, 45, 80), heads=40, name="wan2.2-720p-81f layer (config 3)"),
    2: dict(grid=(21, 30, 52), heads=40, name="wan2.2-480p-81f layer (config 2)"),
}
SPARSE = dict(num_q_centroids=200, num_k_centroids=1000, target_density=0.3, kmeans_iter_init=10,
              probe_rows=64, repair_rank=16, repair_ridge=0.1, selector_policy="attention_mass",
              selector_budget_mode="fixed_density", kmeans_tol=0.0)


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["bf16_tflops_sustained"]), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """Samples SM clocks and throttle reasons through NVML (read-only queries,
    in-process: no subprocess forks that could stall the launching thread)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)
        self.max_mhz = None

    def _run(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(visible.split(",")[self.index]) if visible else self.index
            h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            while not self._stop.is_set():
                sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((sm, reasons))
                self._stop.wait(0.1)
        except Exception as e:  # sampling is best effort; report why it is missing
            self.error = repr(e)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"],
                    "error": getattr(self, "error", None)}
        sm = [s[0] for s in self.samples]
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


ATTN_DRAM_BYTES_PER_HEAD = (272.19e6 + 64.94e6) / 4


def _print_kernel_table(step, q, k, v, dev):
    """Per-kernel device time of one layer (torch profiler, CUDA activity) to stdout.

    A profiling aid: the numbers include profiler overhead and are not bench values."""
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize(dev)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step(q, k, v)
        torch.cuda.synchronize(dev)
    rows = [(e.device_time_total, e.count, e.key) for e in prof.key_averages() if e.device_time_total > 0]
    total = sum(r[0] for r in rows)
    print(f"{'kernel':72s} {'calls':>6s} {'ms':>9s} {'share':>7s}")
    for t, n, name in sorted(rows, reverse=True):
        print(f"{name[:72]:72s} {n:6d} {t / 1e3:9.3f} {100 * t / total:6.1f}%")
    print(f"{'total':72s} {'':6s} {total / 1e3:9.3f}")


def _budget_modes(route, q, k, v, init_rows, cfg, dev, n):
    """The reference's two budget modes (``n8_v6.py:1026-1061``) side by side: the
    shipped fixed density (the timed bench line) and SVG top-p budgets (cumulative
    softmax mass 0.3, the literal reading of "keep 30% of cluster-pair mass"), each
    with its achieved cluster-pair density; the top-p layer is timed eagerly
    (CUDA events, second of two calls).  A side measurement, not the bench value."""
    from sparsepr_b200 import N8V6Config, N8V6Core, sparse_attention
    from sparsepr_b200.attention import kept_flops

    heads = q.shape[1]

    def pair_density(rt):
        pairs = (rt.video_dynamic_map.long() * rt.k_cluster_sizes.long().unsqueeze(1)).sum(-1)
        return float((pairs * rt.q_cluster_sizes.long()).sum().item()) / float(heads * n * n)

    modes = {"fixed_density": {"target_density": SPARSE["target_density"], "pair_density": pair_density(route)}}
    cfg_tp = N8V6Config(**{**SPARSE, "selector_budget_mode": "svg_ear_top_p", "svg_ear_top_p": 0.3})
    for _ in range(2):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        _out, dens, info = sparse_attention(q, k, v, N8V6Core(cfg_tp, init_indices=init_rows))
        e1.record()
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    kept = int(kept_flops(info["route"], 128, cfg.probe_rows, n).item())
    modes["svg_ear_top_p"] = {"top_p": 0.3, "pair_density": pair_density(info["route"]), "reported_density": dens,
                              "ms_eager": ms, "kept_tflops": kept / (ms * 1e-3) / 1e12}
    return modes


def _print_route_reuse(cfg, q, k, v, dev, args):
    """Device time of a refreshed layer call and of a temporal-reuse call
    (cached route, current Q/K/V) through ``RouteCache``; one JSON line.
    A side measurement, not the bench line: the headline step routes fresh."""
    from sparsepr_b200 import N8V6Core, RouteCache, RouteReuseConfig

    cache = RouteCache(RouteReuseConfig(dense_first_steps=0, route_refresh_every=1 << 30))
    core = N8V6Core(cfg)
    times = {"refresh": [], "temporal_reuse": []}
    for i in range(args.warmup + args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if i == 0:
            cache.entries.clear()
        a.record()
        out, _, info = cache.attention(q, k, v, core, module_id=0, step=i)
        b.record()
        torch.cuda.synchronize(dev)
        if i == 0 or i >= args.warmup:
            times[info["route_action"]].append(a.elapsed_time(b))
        del out, info
    print(json.dumps({"route_reuse": {"refresh_ms": times["refresh"][0],
                                      "reuse_ms": statistics.median(times["temporal_reuse"]),
                                      "reuse_calls": len(times["temporal_reuse"]), "heads": q.shape[1]}}))


def run_b200(args):
    import torch.distributed as dist

    from sparsepr_b200 import N8V6Config, N8V6Core, kernels as K, sparse_attention
    from sparsepr_b200.attention import kept_flops
    from sparsepr_b200.graph import ConcurrentSparseAttention, StreamedSparseAttention
    from sparsepr_b200.sharding import head_shard, reduce_step_stats
    from sparsepr_b200.synthetic import random_init_indices, synthetic_qkv_heads

    world, rank, local = _dist()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    cfgd = dict(CONFIGS[args.config])
    if args.heads:
        cfgd["heads"] = args.heads
    heads = cfgd["heads"]
    try:
        h0, h1 = head_shard(heads, world, rank)
    except ValueError as e:
        raise SystemExit(str(e))
    local_heads = h1 - h0
    grid = cfgd["grid"]
    n = grid[0] * grid[1] * grid[2]
    # Synthetic Q/K/V for this rank's heads, generated on the device by global head
    # index (each head has its own seeded generator), so every N processes the same
    # tensors; the cold-start centroid rows are this rank's rows of the all-heads draw.
    q, k, v = synthetic_qkv_heads(h0, h1, 128, grid, dtype=torch.bfloat16, device=dev)
    cfg = N8V6Config(**SPARSE)
    init_rows = (random_init_indices(heads, n, cfg.num_k_centroids, cfg.kmeans_init_seed)[h0:h1].to(dev),
                 random_init_indices(heads, n, cfg.num_q_centroids, cfg.kmeans_init_seed + 1)[h0:h1].to(dev))

    def step(qq, kk, vv, events=None):
        core = N8V6Core(cfg, init_indices=init_rows)  # cold call: full k-means from the seeded init every step
        return sparse_attention(qq, kk, vv, core, attn_events=events)

    for _ in range(args.warmup):
        out, _, info = step(q, k, v)
    torch.cuda.synchronize(dev)
    kept = int(kept_flops(info["route"], 128, cfg.probe_rows, n).item())
    route = info["route"]
    sel_keys = (route.video_dynamic_map.long() * route.k_cluster_sizes.long().unsqueeze(1)).sum(-1)
    attn_flops = int((4 * 128 * (sel_keys * route.q_cluster_sizes.long()).sum()).item())
    del out, info

    if args.kernel_table:
        _print_kernel_table(step, q, k, v, dev)
        return
    if args.route_reuse:
        _print_route_reuse(cfg, q, k, v, dev, args)
        return
    # Both budget modes of the reference, each with its achieved pair density (N = 1 only).
    budget_modes = _budget_modes(route, q, k, v, init_rows, cfg, dev, n) if world == 1 else None
    del route

    # Eager pass: per-kernel events for the attention roofline and the launch count.
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    launches0 = K.LAUNCHES[0]
    t0.record()
    for i in range(args.steps):
        out, _, info = step(q, k, v, ev[i])
        del out, info
    t1.record()
    torch.cuda.synchronize(dev)
    launches = (K.LAUNCHES[0] - launches0) // max(args.steps, 1)
    eager_ms = t0.elapsed_time(t1) / args.steps
    attn_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)

    # Timed region: the whole layer captured as CUDA graphs (all kernels of the
    # step, fresh routing every replay), inputs resident in HBM; the heads run as
    # `--graph-chunks` concurrent graph chains (head ranges on their own streams).
    # Concurrent head-range chains help at many heads per GPU (latency-bound
    # routing kernels of one chain overlap the other's); at a few heads per
    # GPU one chain is faster (measured: 40 heads 2 chains < 1; 5 heads 1 < 2 < 5).
    chains = args.graph_chunks if args.graph_chunks > 0 else (2 if local_heads >= 20 else 1)
    g = ConcurrentSparseAttention(q.shape, cfg, dev, chunks=chains, warmup=max(1, args.warmup),
                                  head_offset=h0, total_heads=heads)
    n_graphs = len(g.graphs)
    g.load(q, k, v)
    g.capture()
    for _ in range(args.warmup):
        g.replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(dev.index) as clocks:
        t0.record()
        for _ in range(args.steps):
            g.replay()
        t1.record()
        torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        dist.barrier()

    # End to end through the public host-buffer API: every step copies this
    # step's pinned host inputs to the device and the output back, streamed in
    # head chunks so the copies of one chunk overlap the compute of another.
    sample = tuple(t[:, :2].cpu() for t in (q, k, v)) if world == 1 else None
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hout = torch.empty(hq.shape, dtype=torch.bfloat16).pin_memory()
    del q, k, v, g
    torch.cuda.synchronize(dev)
    # Heads per streamed chunk: about eight chunks per rank (5 at 40 heads, 1 at
    # 5), so the copies of one chunk overlap the compute of the others.
    chunk = args.e2e_chunk if args.e2e_chunk > 0 else max(1, local_heads // 8)
    while local_heads % chunk:
        chunk -= 1
    sg = StreamedSparseAttention(hq.shape, cfg, dev, heads_per_chunk=chunk, slots=args.e2e_slots,
                                 warmup=max(1, args.warmup)).capture()
    for _ in range(max(1, args.warmup)):
        sg(hq, hk, hv, hout)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(1, args.steps)
    if world > 1:
        dist.barrier()
    e0.record()
    for _ in range(e_steps):
        sg(hq, hk, hv, hout)
    e1.record()
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / e_steps
    del sg
    h2d = 3 * hq.numel() * 2
    d2h = hout.numel() * 2

    (ms, e2e_ms, attn_ms), (kept, attn_flops) = reduce_step_stats([ms, e2e_ms, attn_ms], [kept, attn_flops], dev)
    if world > 1:
        h2d *= world
        d2h *= world
    if rank == 0:
        burst, sustained, hbm, src = _peaks()
        per_rank_attn_flops = attn_flops / world
        achieved = per_rank_attn_flops / (attn_ms * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": kept / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded smooth-field Q/K + noise, V~N(0,1); no public dataset for this path)",
            "config": {"workload": cfgd["name"], "tokens": n, "heads": heads, "head_dim": 128,
                       "heads_per_gpu": local_heads, "q_clusters": 200, "k_clusters": 1000,
                       "lloyd_iters": 10, "keep": "30% of key tokens per query cluster (fixed_density 0.3)",
                       "probe_rows": 64, "repair_rank": 16, "parallelism": f"heads-sharded x{world}",
                       "l2": "inputs (3 x 774 MB bf16 per 40 heads) exceed the 126 MB L2; no flush"},
            "kept_tflop_per_step": kept / 1e12,
            "timing": f"CUDA-graph replay of the whole layer ({n_graphs} concurrent head-range graphs per step); "
                      "eager launches (one stream) in eager_ms_per_step",
            "eager_ms_per_step": eager_ms,
            "e2e": {"value": kept / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "api": f"StreamedSparseAttention, pinned host buffers, {chunk}-head chunks on "
                           f"{args.e2e_slots} streams"},
            "roofline": {"kernel": "block_sparse_attn_kernel", "bound": "tensor", "achieved": achieved,
                         "peak": sustained, "peak_source": f"bf16_tflops_sustained ({src})", "unit": "TFLOP/s",
                         "frac": achieved / sustained,
                         # DRAM bytes per launch: ncu capture of the 4-head case (272 MB read +
                         # 65 MB written), scaled by heads (inputs and output are read/written once).
                         "traffic": ATTN_DRAM_BYTES_PER_HEAD * local_heads, "traffic_source": "ncu, 4-head capture scaled",
                         "attn_ms": attn_ms,
                         "attn_share_of_step": attn_ms / ms},
            "gpu_launches": int(launches),
            "budget_modes": budget_modes,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args, heads_sample=2, qkv=sample)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_ulysses(args):
    """Sequence-sharded variant (N > 1): each rank holds ``[1, N/W, H, D]`` of Q, K, V; per step
    an NCCL all-to-all regroups them into head shards, the layer runs on the local heads and a
    second all-to-all returns the output to sequence shards.  One JSON line (not the bench
    line): step ms (max over ranks), the exchange's share, and an exactness check of the
    exchange against direct head slices of the same tensors."""
    import torch.distributed as dist

    from sparsepr_b200 import N8V6Config, N8V6Core
    from sparsepr_b200.sharding import reduce_step_stats
    from sparsepr_b200.synthetic import synthetic_qkv
    from sparsepr_b200.ulysses import UlyssesSparseAttention, head_to_seq, seq_to_head

    world, rank, local = _dist()
    if world < 2:
        raise SystemExit("--ulysses needs torchrun with 2 or more ranks")
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    cfgd = CONFIGS[args.config]
    grid, heads = cfgd["grid"], cfgd["heads"]
    n = grid[0] * grid[1] * grid[2]
    ns, hs = n // world, heads // world
    # Every rank draws the same full tensors and keeps its sequence shard (BLHD).
    full = synthetic_qkv(heads, 128, grid, dtype=torch.bfloat16, device=dev, seeds=(0, 1, 2))
    shards = [t.permute(0, 2, 1, 3)[:, rank * ns:(rank + 1) * ns].contiguous() for t in full]
    exact = all(torch.equal(seq_to_head(x), t[:, rank * hs:(rank + 1) * hs]) for x, t in zip(shards, full))
    exact = exact and torch.equal(head_to_seq(seq_to_head(shards[0])), shards[0])
    del full
    layer = UlyssesSparseAttention(N8V6Config(**SPARSE))
    inner = layer.attention
    ev = []

    def timed(q, k, v):  # the head-local layer, bracketed to separate it from the exchange
        layer.core = N8V6Core(layer.core.config)  # cold call each step, like the bench line
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        o = inner(q, k, v)
        b.record()
        ev.append((a, b))
        return o

    layer.attention = timed
    for _ in range(args.warmup):
        layer(*shards)
    torch.cuda.synchronize(dev)
    ev.clear()
    dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        out = layer(*shards)
    t1.record()
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / args.steps
    layer_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    (ms, layer_ms), (ok,) = reduce_step_stats([ms, layer_ms], [0.0 if exact else 1.0], dev)
    if rank == 0:
        print(json.dumps({"ulysses": {
            "n_gpus": world, "config": cfgd["name"], "tokens_per_rank": ns, "heads_per_rank": hs,
            "ms_per_step": ms, "head_local_layer_ms": layer_ms, "exchange_ms": ms - layer_ms,
            "exchange_bytes_per_rank": int(4 * 2 * ns * heads * 128 * (world - 1) / world),
            "exchange_exact": ok == 0.0, "out_shape": list(out.shape), "timing": "eager, CUDA events, max over ranks"}}),
            flush=True)
    dist.destroy_process_group()


def run_dit(args):
    """Config 4: one denoising step of a random-init HunyuanVideo-architecture DiT
    (hidden 3072, 24 x 128 heads, 20 double + 40 single blocks, bf16) on a 720p /
    129-frame latent (33 x 45 x 80 = 118,800 video tokens) plus 256 text tokens, with
    SparsePR (svg_ear_value scores, config-3 settings) on the video tokens of every
    block.  N > 1 ranks shard the video tokens (Ulysses exchange around attention).
    One JSON line (not the bench line)."""
    import torch.distributed as dist

    from sparsepr_b200 import N8V6Config
    from sparsepr_b200.hunyuan_dit import HunyuanDiT, HunyuanDiTConfig, JointAttention, SparsePRBlocks
    from sparsepr_b200.sharding import reduce_step_stats

    world, rank, local = _dist()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    cfg = HunyuanDiTConfig()
    model = HunyuanDiT(cfg, dev, seed=0)  # same seed on every rank: same weights
    params = sum(w.numel() for w in _dit_tensors(model))
    g = torch.Generator(device=dev).manual_seed(1)
    latent = torch.randn(cfg.in_channels, 33, 90, 160, device=dev, generator=g)
    text = torch.randn(256, cfg.text_dim, device=dev, generator=g)
    pooled = torch.randn(cfg.vec_dim, device=dev, generator=g)
    t, guidance = torch.tensor(900.0, device=dev), torch.tensor(6.0, device=dev)
    sp = N8V6Config(**{**SPARSE, "selector_policy": "svg_ear_value"})
    blocks = SparsePRBlocks(sp, cfg.double_blocks + cfg.single_blocks, prompt_length=256)
    events = []
    att = JointAttention(blocks, events=events)

    def step():
        blocks.reset()  # cold routing in every block, as on the first denoising step
        return model.forward(latent, text, t, pooled, guidance, att, rank=rank, world=world)

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    events.clear()
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, args.steps)
    with ClockSampler(dev.index) as clocks:
        t0.record()
        for _ in range(steps):
            out = step()
        t1.record()
        torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / steps
    attn_ms = sum(a.elapsed_time(b) for a, b in events) / steps
    (ms, attn_ms), _ = reduce_step_stats([ms, attn_ms], [0.0], dev)
    if rank == 0:
        n_video = 33 * 45 * 80
        print(json.dumps({"dit": {
            "workload": "HunyuanVideo-architecture DiT, one denoising step (config 4)", "n_gpus": world,
            "ms_per_step": ms, "sparsepr_attention_ms": attn_ms, "attention_share": attn_ms / ms,
            "video_tokens": n_video, "text_tokens": 256, "heads": cfg.heads, "blocks": cfg.double_blocks + cfg.single_blocks,
            "params": params, "parallelism": f"video tokens sequence-sharded x{world} (Ulysses)" if world > 1 else "1 GPU",
            "sparsepr": "svg_ear_value, 200/1000 clusters, 10 Lloyd iterations, keep 30%, repair (64 probes, rank 16)",
            "data": "random-init bf16 weights, latent ~ N(0,1), text ~ N(0,1)", "out_tokens_per_rank": int(out.shape[0]),
            "timing": "eager, CUDA events, max over ranks", "steps": steps, "clocks": clocks.summary()}}), flush=True)
    if world > 1:
        dist.destroy_process_group()


def _dit_tensors(model):
    def walk(x):
        if isinstance(x, torch.Tensor):
            yield x
        elif isinstance(x, (list, tuple)):
            for y in x:
                yield from walk(y)
        elif isinstance(x, dict):
            for y in x.values():
                yield from walk(y)

    for name, val in vars(model).items():
        if name not in ("cfg", "device", "dtype"):
            yield from walk(val)


def run_kmeans(args):
    """Config 1: standalone batched k-means (the flash_kmeans workload): 40 problems x
    75,600 points x 128 bf16, K=256, 10 Lloyd iterations from seeded k-means++ centroids,
    tol=0.  One JSON line (a side bench, not the layer line): ms per 10-iteration run,
    TFLOP/s with the reference self-bench's count 2*B*N*D*K*iters
    (``flash_kmeans/kmeans_triton_impl.py:199-261``), and the device time split into
    the assignment GEMM and the sort + centroid update, each against its roofline."""
    from sparsepr_b200 import batch_kmeans_Euclid
    from sparsepr_b200.synthetic import kmeans_plus_plus, synthetic_kmeans_points

    world, rank, local = _dist()
    dev = torch.device("cuda", local if world > 1 else 0)
    b, grid, k, iters, d = (args.heads or 40), (21, 45, 80), 256, 10, 128
    n = grid[0] * grid[1] * grid[2]
    x = synthetic_kmeans_points(b, d, grid, 256, device=dev, seed=0)
    init = kmeans_plus_plus(x, k, seed=3)
    torch.cuda.synchronize(dev)

    def run():
        return batch_kmeans_Euclid(x, k, max_iters=iters, tol=0.0, init_centroids=init, round_centroids_to_input=True)

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        t0.record()
        for _ in range(args.steps):
            labels, cent, sizes, it = run()
        t1.record()
        torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / args.steps
    flops = 2.0 * b * n * d * k * iters
    # Split of one run's device time between the assignment GEMM and the rest
    # (label sort, centroid update, norms) from the torch profiler: a share, not a bench value.
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        run()
        torch.cuda.synchronize(dev)
    times = [(e.key, e.device_time_total) for e in prof.key_averages() if e.device_time_total > 0]
    total_us = sum(t for _, t in times)
    assign_us = sum(t for name, t in times if "assign" in name)
    assign_ms = ms * assign_us / max(total_us, 1e-9)
    burst, sustained, hbm, src = _peaks()
    upd_bytes = iters * (x.numel() * 2 + b * n * 4 * 3)  # per iteration: X read once, labels + order
    line = {"kmeans": {
        "workload": "standalone batched k-means (config 1)", "problems": b, "points": n, "dim": d, "k": k,
        "iters": iters, "dtype": "bf16 points, fp32 distances (TF32-exact on bf16 values), bf16 centroids",
        "ms_per_run": ms, "tflops": flops / (ms * 1e-3) / 1e12,
        "assign_ms_per_run": assign_ms, "assign_tflops": flops / (assign_ms * 1e-3) / 1e12,
        "split": "assignment share of one run's device time (torch profiler), applied to ms_per_run",
        "update_ms_per_run": ms - assign_ms,
        "update_gbs": upd_bytes / ((ms - assign_ms) * 1e-3) / 1e9, "hbm_peak_gbs": hbm,
        "bf16_peak_tflops": burst, "peak_source": src, "steps": args.steps, "warmup": args.warmup,
        "data": "synthetic smooth mixture of 256 Gaussians on 21x45x80, seeded k-means++ init",
        "clocks": clocks.summary()}}
    if not args.no_cpu_baseline:
        import oracle

        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        xs, cs = x[:1].cpu(), init[:1].cpu()
        t = time.perf_counter()
        oracle.batch_kmeans_euclid(xs, k, 2, 0.0, cs)
        dt = time.perf_counter() - t
        line["kmeans"]["cpu_baseline"] = {
            "value": 2.0 * n * d * k * 2 / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"1 of {b} problems, 2 of {iters} iterations, {dt:.1f} s"}
    print(json.dumps(line), flush=True)


def cpu_baseline(args, heads_sample: int = 2, qkv=None):
    """The oracle (CPU restatement of the reference algorithm) on a bounded sample:
    the same layer on heads 0..``heads_sample``-1 of the bench's own inputs
    (``qkv``, else generated like them), scaled to kept TFLOP/s."""
    import types

    import oracle
    from sparsepr_b200.synthetic import synthetic_qkv_heads

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfgd = CONFIGS[args.config]
    grid = cfgd["grid"]
    n = grid[0] * grid[1] * grid[2]
    if qkv is None:  # the GPU arm generates on the device: use the same generator where there is one
        gen_dev = torch.device("cuda", 0) if torch.cuda.is_available() else None
        qkv = tuple(t.cpu() for t in synthetic_qkv_heads(0, heads_sample, 128, grid, device=gen_dev))
    q, k, v = (t[:, :heads_sample] for t in qkv)
    oc = types.SimpleNamespace(role_q_rank=64, role_k_rank=48, metric_sample_tokens=2048, repair_alpha=1.0,
                               repair_norm_cap=0.0, svg_ear_top_p=0.85, adaptive_budget_min_density=0.0,
                               adaptive_budget_max_density=1.0, **SPARSE)
    t = time.perf_counter()
    _out, r, _base, _ = oracle.oracle_sparse_attention(q, k, v, oc, init_seed=0, tol=0.0)
    dt = time.perf_counter() - t
    kept = 4 * 128 * (oracle.kept_pairs(r.mask, r.q_sizes, r.k_sizes) + heads_sample * SPARSE["probe_rows"] * n)
    return {"value": kept / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{heads_sample} of {cfgd['heads']} heads of {cfgd['name']}, full route+attention+repair, "
                      f"{dt:.1f} s", "seconds": dt, "ms_per_layer_extrapolated": dt * 1e3 * cfgd["heads"] / heads_sample}


def run_reference(args):
    """The reference algorithm's CPU path (the oracle port) on the box's host cores.
    Each step is one bounded sample: heads 0-1 of the bench's inputs, the whole layer
    (route, attention, repair); ``ms_per_step`` is that sample's measured time and
    the 40-head extrapolation is reported beside it."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    cfgd = CONFIGS[args.config]
    grid = cfgd["grid"]
    gen_dev = torch.device("cuda", 0) if torch.cuda.is_available() else None
    from sparsepr_b200.synthetic import synthetic_qkv_heads

    qkv = tuple(t.cpu() for t in synthetic_qkv_heads(0, 2, 128, grid, device=gen_dev))
    res = [cpu_baseline(args, heads_sample=2, qkv=qkv) for _ in range(args.warmup + args.steps)]
    timed = res[args.warmup:]
    v = statistics.median(x["value"] for x in timed)
    cb = dict(timed[-1])
    cb["value"] = v
    sample_ms = statistics.median(x["seconds"] for x in timed) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sample_ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32 (CPU)", "data": "synthetic",
        "step": "one bounded sample: 2 of the 40 heads, full layer",
        "ms_per_layer_extrapolated": sample_ms * cfgd["heads"] / 2,
        "config": {"workload": cfgd["name"], "tokens": cfgd["grid"][0] * cfgd["grid"][1] * cfgd["grid"][2],
                   "heads": cfgd["heads"], "sample_heads": 2},
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", type=int, default=3, choices=sorted(CONFIGS) + [1, 4],
                    help="3 (default) or 2: the SparsePR layer; 1: standalone batched k-means; "
                         "4: a HunyuanVideo-architecture DiT step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--heads", type=int, default=0, help="override the head count (profiling runs)")
    ap.add_argument("--graph-chunks", type=int, default=0,
                    help="concurrent head-range graphs of the timed layer (1 = one graph for all heads; "
                         "0: 2 at 20 or more heads per GPU, else 1)")
    ap.add_argument("--e2e-chunk", type=int, default=0,
                    help="heads per streamed chunk in the e2e measurement (0: about eight chunks per rank)")
    ap.add_argument("--e2e-slots", type=int, default=8, help="concurrent graph slots (streams) in the e2e measurement")
    ap.add_argument("--ulysses", action="store_true",
                    help="(torchrun, N > 1) time the sequence-sharded Ulysses variant instead of the bench line")
    ap.add_argument("--route-reuse", action="store_true",
                    help="time a refreshed and a cached-route (temporal reuse) layer call instead of the bench line")
    ap.add_argument("--kernel-table", action="store_true",
                    help="print per-kernel device times of one layer (torch profiler) instead of the bench line")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.ulysses:
        run_ulysses(args)
    elif args.config == 4:
        run_dit(args)
    elif args.config == 1:
        run_kmeans(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
