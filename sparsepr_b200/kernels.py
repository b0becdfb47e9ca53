"""Torch-tensor wrappers over the C ABI (device memory and streams come from PyTorch).

Every function checks shapes/dtypes/devices, allocates its outputs with
``torch.empty`` on the input's device, and launches on the current CUDA
stream.  There is no CPU path: non-CUDA inputs raise ``RuntimeError``.
"""

from __future__ import annotations

import contextlib

import torch

from . import _lib

_DT = {torch.float32: _lib.SPR_F32, torch.bfloat16: _lib.SPR_BF16, torch.float16: _lib.SPR_F16}
_WS: dict[tuple, torch.Tensor] = {}

# Number of sparsepr_b200 kernels launched through this module (per process);
# bench.py reports the count inside its timed region.
LAUNCHES = [0]


def _count(n: int) -> None:
    LAUNCHES[0] += int(n)


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _cuda(*ts: torch.Tensor) -> torch.device:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"sparsepr_b200 kernels need CUDA tensors, got a {t.device} tensor")
    return ts[0].device


def _contig(name: str, t: torch.Tensor) -> torch.Tensor:
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous, got strides {t.stride()}")
    return t


_SCOPE = [""]


@contextlib.contextmanager
def workspace_scope(name: str):
    """Workspaces requested inside the block are private to ``name``.

    Work that may run concurrently (two captured graphs replayed on different
    streams) must not share scratch buffers; each graph captures under its own
    scope."""
    prev = _SCOPE[0]
    _SCOPE[0] = name
    try:
        yield
    finally:
        _SCOPE[0] = prev


def workspace(dev: torch.device, nbytes: int, tag: str = "default") -> torch.Tensor:
    """Caller-owned scratch, cached per (device, scope, tag) and grown on demand."""
    key = (dev.type, dev.index, _SCOPE[0], tag)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)
        _WS[key] = buf
    return buf


def _precision(p: str) -> int:
    if p not in _lib.PRECISION:
        raise ValueError(f"k-means precision must be one of {sorted(_lib.PRECISION)}, got {p!r}")
    return _lib.PRECISION[p]


def kmeans_assign(x: torch.Tensor, centroids: torch.Tensor, precision: str = "tf32") -> torch.Tensor:
    """Nearest centroid per point (ties -> lowest index): x [B,N,D], c [B,K,D] fp32 -> int32 [B,N].

    ``precision``: "tf32" (tensor-core TF32 dot products, the reference GPU
    behaviour) or "fp32" (3xTF32, fp32-accurate, d <= 64)."""
    dev = _cuda(x, centroids)
    b, n, d = x.shape
    k = centroids.shape[1]
    if centroids.shape != (b, k, d) or centroids.dtype != torch.float32:
        raise RuntimeError(f"centroids must be fp32 [B,K,D]={b, k, d}, got {tuple(centroids.shape)} {centroids.dtype}")
    labels = torch.empty((b, n), dtype=torch.int32, device=dev)
    nbytes = _lib.query("spr_kmeans_workspace_bytes", b, n, d, k)
    ws = workspace(dev, nbytes, "kmeans")
    _count(1)
    _lib.call("spr_kmeans_assign", _p(_contig("x", x)), _DT[x.dtype], b, n, d, k, _p(_contig("centroids", centroids)),
              _precision(precision), _p(labels), _p(ws), ws.numel(), _stream(dev))
    return labels


def kmeans_error_code(dev: torch.device) -> int:
    """Device status word of the last k-means call on ``dev`` (0 = ok).  Synchronises; for tests."""
    ws = _WS.get((dev.type, dev.index, _SCOPE[0], "kmeans"))
    if ws is None:
        return 0
    torch.cuda.synchronize(dev)
    return int(ws[:4].view(torch.int32).item())


def kmeans_lloyd(x: torch.Tensor, init_centroids: torch.Tensor, iters: int, tol: float = 0.0,
                 round_centroids_to_input: bool = False, precision: str = "tf32"):
    """Batched Lloyd k-means with an on-device ``tol`` stop.

    Returns ``(labels i32 [B,N], centroids f32 [B,K,D], sizes i32 [B,K],
    offsets i32 [B,K+1], order i32 [B,N], iters_done i32 [1] device tensor)``.
    """
    dev = _cuda(x, init_centroids)
    b, n, d = x.shape
    k = init_centroids.shape[1]
    if init_centroids.shape != (b, k, d):
        raise RuntimeError(f"init centroids must be [B,K,D]={b, k, d}, got {tuple(init_centroids.shape)}")
    cent = init_centroids.to(torch.float32).contiguous().clone()
    labels = torch.empty((b, n), dtype=torch.int32, device=dev)
    sizes = torch.empty((b, k), dtype=torch.int32, device=dev)
    offsets = torch.empty((b, k + 1), dtype=torch.int32, device=dev)
    order = torch.empty((b, n), dtype=torch.int32, device=dev)
    iters_done = torch.zeros((1,), dtype=torch.int32, device=dev)
    nbytes = _lib.query("spr_kmeans_workspace_bytes", b, n, d, k)
    ws = workspace(dev, nbytes, "kmeans")
    rd = _DT[x.dtype] if round_centroids_to_input else _lib.SPR_F32
    _count(6 * int(iters))
    _lib.call("spr_kmeans_lloyd", _p(_contig("x", x)), _DT[x.dtype], b, n, d, k, int(iters), float(tol), rd,
              _precision(precision),
              _p(cent), _p(labels), _p(sizes), _p(offsets), _p(order), _p(iters_done), _p(ws), ws.numel(),
              _stream(dev))
    return labels, cent, sizes, offsets, order, iters_done


def label_sort(labels: torch.Tensor, k: int):
    """Stable counting sort: (sizes i32 [B,K], offsets i32 [B,K+1], order i32 [B,N])."""
    dev = _cuda(labels)
    if labels.dtype != torch.int32:
        raise RuntimeError("labels must be int32")
    b, n = labels.shape
    sizes = torch.empty((b, k), dtype=torch.int32, device=dev)
    offsets = torch.empty((b, k + 1), dtype=torch.int32, device=dev)
    order = torch.empty((b, n), dtype=torch.int32, device=dev)
    nbytes = _lib.query("spr_kmeans_workspace_bytes", b, n, 16, k)
    ws = workspace(dev, nbytes, "kmeans")
    _count(3)
    _lib.call("spr_label_sort", _p(_contig("labels", labels)), b, n, k, _p(sizes), _p(offsets), _p(order), _p(ws),
              ws.numel(), _stream(dev))
    return sizes, offsets, order


def centroid_means(x: torch.Tensor, order: torch.Tensor, offsets: torch.Tensor, k: int,
                   fallback: torch.Tensor | None = None, permute: bool = False):
    """Per-cluster fp32 means over the sorted order, optionally emitting the permuted x."""
    dev = _cuda(x, order, offsets)
    b, n, d = x.shape
    means = torch.empty((b, k, d), dtype=torch.float32, device=dev)
    x_perm = torch.empty_like(x) if permute else None
    if fallback is not None:
        fallback = fallback.to(torch.float32).contiguous()
        if fallback.shape != (b, k, d):
            raise RuntimeError(f"fallback must be [B,K,D]={b, k, d}")
    _count(1)
    _lib.call("spr_centroid_means", _p(_contig("x", x)), _DT[x.dtype], _p(order), _p(offsets), b, n, d, k,
              _p(fallback), _p(means), _p(x_perm), _stream(dev))
    return means, x_perm


def permute_rows(x: torch.Tensor, idx: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    """Gather ``y[b,s]=x[b,idx[b,s]]`` (or scatter when ``inverse``) over [B,N,D] rows."""
    dev = _cuda(x, idx)
    b, n, d = x.shape
    y = torch.empty_like(x)
    _count(1)
    _lib.call("spr_permute_rows", _p(_contig("x", x)), _p(_contig("idx", idx)), _p(y), b, n, d, x.element_size(),
              int(inverse), _stream(dev))
    return y


def attention_mass_scores(q_centroids: torch.Tensor, k_sorted: torch.Tensor, k_offsets: torch.Tensor) -> torch.Tensor:
    """log-sum-exp attention mass per (query centroid, key cluster) -> fp32 [B,Cq,Ck]."""
    dev = _cuda(q_centroids, k_sorted, k_offsets)
    b, cq, d = q_centroids.shape
    ck = k_offsets.shape[1] - 1
    n = k_sorted.shape[1]
    if k_sorted.dtype != torch.bfloat16:
        raise RuntimeError("k_sorted must be bf16")
    qc = q_centroids.float().contiguous()
    scores = torch.empty((b, cq, ck), dtype=torch.float32, device=dev)
    _count(1)
    _lib.call("spr_attention_mass_scores", _p(qc), _p(_contig("k_sorted", k_sorted)),
              _p(_contig("k_offsets", k_offsets)), b, cq, ck, n, d, _p(scores), _stream(dev))
    return scores


def svg_ear_value_scores(q_centroids: torch.Tensor, k_sorted: torch.Tensor, v_sorted: torch.Tensor,
                         k_centroids: torch.Tensor, v_centroids: torch.Tensor, k_offsets: torch.Tensor) -> torch.Tensor:
    """SVG-EAR value-error selector scores -> fp32 [B,Cq,Ck] (-inf for empty key clusters)."""
    dev = _cuda(q_centroids, k_sorted, v_sorted, k_centroids, v_centroids, k_offsets)
    b, cq, d = q_centroids.shape
    ck = k_offsets.shape[1] - 1
    n = k_sorted.shape[1]
    if k_sorted.dtype != torch.bfloat16 or v_sorted.dtype != torch.bfloat16:
        raise RuntimeError("k_sorted and v_sorted must be bf16")
    if v_sorted.shape != k_sorted.shape or tuple(k_centroids.shape) != (b, ck, d) or \
            tuple(v_centroids.shape) != (b, ck, d):
        raise RuntimeError(f"SVG-EAR shapes: k {tuple(k_sorted.shape)}, v {tuple(v_sorted.shape)}, "
                           f"kc {tuple(k_centroids.shape)}, vc {tuple(v_centroids.shape)}, ck={ck}")
    qc = q_centroids.float().contiguous()
    kc = k_centroids.float().contiguous()
    vc = v_centroids.float().contiguous()
    scores = torch.empty((b, cq, ck), dtype=torch.float32, device=dev)
    nbytes = _lib.query("spr_svg_ear_value_scores_workspace_bytes", b, cq, ck, n)
    ws = workspace(dev, nbytes, "svg_ear")
    _count(3)
    _lib.call("spr_svg_ear_value_scores", _p(qc), _p(_contig("k_sorted", k_sorted)),
              _p(_contig("v_sorted", v_sorted)), _p(kc), _p(vc), _p(_contig("k_offsets", k_offsets)), b, cq, ck, n,
              d, _p(scores), _p(ws), ws.numel(), _stream(dev))
    return scores


def role_projection(x: torch.Tensor, factor: torch.Tensor, mode: str) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Role features of bf16 tokens x [B,N,128] with factor [B,128,r] (tensor cores, fp32 accuracy).

    ``mode="global"``: divided by one RMS per problem, returns ``(feat, scale [B,1,1])``
    (the K role); ``mode="row"``: divided by each row's RMS, returns ``(feat, None)``
    (the Q role)."""
    dev = _cuda(x, factor)
    if x.dtype != torch.bfloat16 or x.dim() != 3:
        raise RuntimeError(f"role projection expects bf16 [B,N,D] tokens, got {x.dtype} {tuple(x.shape)}")
    b, n, d = x.shape
    r = factor.shape[-1]
    if tuple(factor.shape) != (b, d, r):
        raise RuntimeError(f"role projection factor {tuple(factor.shape)} does not match tokens {tuple(x.shape)}")
    if mode not in ("global", "row"):
        raise ValueError(f"role projection mode must be 'global' or 'row', got {mode!r}")
    f = factor.float().contiguous()
    out = torch.empty((b, n, r), dtype=torch.float32, device=dev)
    scale = torch.empty((b,), dtype=torch.float32, device=dev) if mode == "global" else None
    nbytes = _lib.query("spr_role_projection_workspace_bytes", b, n, r)
    ws = workspace(dev, nbytes, "role_projection")
    _count(4 if mode == "global" else 2)
    _lib.call("spr_role_projection", _p(_contig("x", x)), _p(f), b, n, d, r, 0 if mode == "global" else 1, _p(out),
              _p(scale) if scale is not None else None, _p(ws), ws.numel(), _stream(dev))
    return out, (scale.view(b, 1, 1) if scale is not None else None)


def probe_representatives(feat: torch.Tensor, order: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
    """Per (problem, cluster) the token nearest to the cluster's mean role feature
    -> int32 [B,K] (N for an empty cluster); ``order``/``offsets`` from the k-means sort."""
    dev = _cuda(feat, order, offsets)
    b, n, r = feat.shape
    k = offsets.shape[1] - 1
    if tuple(order.shape) != (b, n) or order.dtype != torch.int32 or offsets.dtype != torch.int32:
        raise RuntimeError(f"probe representatives: order {tuple(order.shape)} {order.dtype}, "
                           f"offsets {tuple(offsets.shape)} {offsets.dtype} for features {tuple(feat.shape)}")
    best = torch.empty((b, k), dtype=torch.int32, device=dev)
    _count(1)
    _lib.call("spr_probe_representatives", _p(_contig("feat", feat.float())), _p(_contig("order", order)),
              _p(_contig("offsets", offsets)), b, n, r, k, _p(best), _stream(dev))
    return best


def role_projection_error_code() -> int:
    """Status word of the last role projection launch (0 = ok; synchronises)."""
    import ctypes

    v = ctypes.c_int(0)
    _lib.call("spr_role_projection_status", ctypes.addressof(v))
    return v.value


def scores_error_code() -> int:
    """Status word of the last attention-mass scores launch (0 = ok; synchronises)."""
    import ctypes

    v = ctypes.c_int(0)
    _lib.call("spr_attention_mass_scores_status", ctypes.addressof(v))
    return v.value


def select_budget(scores: torch.Tensor, k_sizes: torch.Tensor, budgets: torch.Tensor):
    """Budgeted selection -> (routed bool [B,Cq+1,Ck+1], sel_ids i32 [B,Cq,Ck], sel_counts i32 [B,Cq])."""
    dev = _cuda(scores, k_sizes, budgets)
    b, cq, ck = scores.shape
    routed = torch.empty((b, cq + 1, ck + 1), dtype=torch.bool, device=dev)
    ids = torch.empty((b, cq, ck), dtype=torch.int32, device=dev)
    counts = torch.empty((b, cq), dtype=torch.int32, device=dev)
    ks = k_sizes.to(torch.int32).contiguous()
    bu = budgets.to(torch.int32).contiguous()
    _count(1)
    _lib.call("spr_select_budget", _p(_contig("scores", scores)), _p(ks), _p(bu), b, cq, ck, _p(routed), _p(ids),
              _p(counts), _stream(dev))
    return routed, ids, counts


def block_sparse_attention(q_perm, k_perm, v_perm, q_offsets, k_offsets, sel_ids, sel_counts,
                           q_order: torch.Tensor | None = None, out: torch.Tensor | None = None,
                           _ws_tag: str = "attn", repair=None) -> torch.Tensor:
    """Block-sparse attention over kept cluster pairs (bf16, d=128) -> [B,Nq,D] bf16.

    ``repair`` (optional) = ``(state, alpha, probe_rows, probe_dense)`` with
    ``state = (x_mean, x_scale, y_mean, left, basis)`` (rank 16): the repair is
    applied in the kernel's epilogue and the probe rows are stored as their
    dense rows (``probe_rows`` [B,M] token ids in any order, ``probe_dense``
    [B,M,D] bf16)."""
    dev = _cuda(q_perm, k_perm, v_perm, q_offsets, k_offsets, sel_ids, sel_counts)
    b, nq, d = q_perm.shape
    nk = k_perm.shape[1]
    cq = q_offsets.shape[1] - 1
    ck = k_offsets.shape[1] - 1
    for name, t in (("q_perm", q_perm), ("k_perm", k_perm), ("v_perm", v_perm)):
        if t.dtype != torch.bfloat16:
            raise RuntimeError(f"{name} must be bf16, got {t.dtype}")
        _contig(name, t)
    if out is None:
        out = torch.empty_like(q_perm)
    nbytes = _lib.query("spr_block_sparse_attn_workspace_bytes", b, nq, cq)
    ws = workspace(dev, nbytes, _ws_tag)
    rs = None
    keep = ()
    if repair is not None:
        import ctypes

        state, alpha, rows, dense = repair
        xm, xs, ym, left, basis = (t.to(torch.float32).contiguous() for t in state)
        if left.shape[-1] != 16 or left.shape[0] != b:
            raise RuntimeError(f"fused repair needs rank-16 state for {b} problems, got left {tuple(left.shape)}")
        # The kernel looks probe tokens up by binary search: ascending order.
        srt, perm = torch.sort(rows.to(torch.int32), dim=1)
        dense_s = torch.gather(dense.to(torch.bfloat16), 1, perm.unsqueeze(-1).expand(-1, -1, d)).contiguous()
        srt = srt.contiguous()
        keep = (xm, xs, ym, left, basis, srt, dense_s)
        rs = _lib.SprRepairState(_p(xm), _p(xs), _p(ym), _p(left), _p(basis), 16, float(alpha), _p(srt),
                                 _p(dense_s), int(srt.shape[1]))
        _count(1)
    _count(2)
    _lib.call("spr_block_sparse_attn", _p(q_perm), _p(k_perm), _p(v_perm), _p(q_offsets), _p(k_offsets), _p(sel_ids),
              _p(sel_counts), b, nq, nk, d, cq, ck, _p(q_order), None if rs is None else ctypes.byref(rs), _p(out),
              _p(ws), ws.numel(), _stream(dev))
    del keep  # the launch is enqueued; the caching allocator keeps the memory stream-ordered
    return out


def probe_rows_attention(q, k_perm, v_perm, k_offsets, routed, rows, row_cluster):
    """The probe pre-pass of the fused repair: ``(dense [B,M,D], base [B,M,D])`` bf16
    for probe rows ``rows`` [B,M] of the original-order ``q`` [B,N,D]: exact
    attention against all keys, and attention restricted to the key clusters
    that ``routed`` [B,Cq+1,Ck+1] keeps for their query clusters ``row_cluster``."""
    dev = _cuda(q, k_perm, v_perm, k_offsets, routed, rows, row_cluster)
    b, n, d = q.shape
    nk = k_perm.shape[1]
    m = rows.shape[1]
    cq, ck = routed.shape[1] - 1, routed.shape[2] - 1
    for name, t in (("q", q), ("k_perm", k_perm), ("v_perm", v_perm)):
        if t.dtype != torch.bfloat16:
            raise RuntimeError(f"{name} must be bf16, got {t.dtype}")
        _contig(name, t)
    dense = torch.empty((b, m, d), dtype=torch.bfloat16, device=dev)
    base = torch.empty_like(dense)
    ws = workspace(dev, _lib.query("spr_probe_rows_attn_workspace_bytes", b, nk, m), "attn_probe")
    ri = rows.to(torch.int32).contiguous()
    rc = row_cluster.to(torch.int32).contiguous()
    mp = routed.contiguous().view(torch.uint8)
    _count(2)
    _lib.call("spr_probe_rows_attn", _p(q), _p(k_perm), _p(v_perm), _p(_contig("k_offsets", k_offsets)), _p(mp),
              _p(ri), _p(rc), b, n, nk, d, cq, ck, m, _p(dense), _p(base), _p(ws), ws.numel(), _stream(dev))
    return dense, base


# Per device: (device int32[5] snapshot, pinned host copy, event of the copy).
_STATUS: dict[tuple, tuple] = {}
STATUS_WORDS = ("kmeans", "attention", "dense_rows", "role_projection", "attention_mass_scores", "probe_rows")


def collect_status(dev: torch.device) -> None:
    """Stream-ordered snapshot of the device status words of the last calls on
    ``dev`` (k-means, attention, dense probe rows, role projection, scores) into
    pinned host memory; no synchronisation.  :func:`raise_device_status` reads
    it once the copy has landed.  Skipped while a CUDA graph is being captured."""
    if torch.cuda.is_current_stream_capturing():
        return
    key = (dev.type, dev.index)
    entry = _STATUS.get(key)
    if entry is None:
        entry = (torch.zeros(len(STATUS_WORDS), dtype=torch.int32, device=dev),
                 torch.zeros(len(STATUS_WORDS), dtype=torch.int32).pin_memory(), torch.cuda.Event())
        _STATUS[key] = entry
    buf, host, ev = entry
    buf.zero_()
    for i, tag in enumerate(("kmeans", "attn", "attn_dense")):
        ws = _WS.get((dev.type, dev.index, _SCOPE[0], tag))
        if ws is not None:
            buf[i:i + 1].copy_(ws[:4].view(torch.int32))
    st = _stream(dev)
    _lib.call("spr_role_projection_status_async", buf[3:4].data_ptr(), st)
    _lib.call("spr_attention_mass_scores_status_async", buf[4:5].data_ptr(), st)
    ws = _WS.get((dev.type, dev.index, _SCOPE[0], "attn_probe"))
    if ws is not None:
        buf[5:6].copy_(ws[:4].view(torch.int32))
    host.copy_(buf, non_blocking=True)
    ev.record()


def raise_device_status(dev: torch.device, wait: bool = False) -> None:
    """Raise ``RuntimeError`` if the last snapshot of :func:`collect_status` on
    ``dev`` holds a non-zero status word (a device-side bounded wait gave up, so
    that call's output is incomplete).  Without ``wait`` a snapshot still in
    flight is left for a later check."""
    entry = _STATUS.get((dev.type, dev.index))
    if entry is None or torch.cuda.is_current_stream_capturing():
        return
    _buf, host, ev = entry
    if wait:
        ev.synchronize()
    elif not ev.query():
        return
    words = host.tolist()
    if any(words):
        bad = {name: w for name, w in zip(STATUS_WORDS, words) if w}
        host.zero_()
        raise RuntimeError(f"sparsepr_b200 device status words are non-zero (a bounded device wait gave up; "
                           f"the output of that call is incomplete): {bad}")


def attention_error_code(dev: torch.device) -> int:
    """Device status word of the last block-sparse attention launch on ``dev``
    (0 = ok, else the bounded wait that gave up).  Synchronises; for tests."""
    ws = _WS.get((dev.type, dev.index, _SCOPE[0], "attn"))
    if ws is None:
        return 0
    torch.cuda.synchronize(dev)
    return int(ws[:4].view(torch.int32).item())


def dense_attention_rows(q_rows: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Exact attention of [B,M,D] query rows against all [B,N,D] keys (one cluster pair)."""
    dev = _cuda(q_rows, k, v)
    b, m, _ = q_rows.shape
    n = k.shape[1]
    two = torch.arange(2, dtype=torch.int32, device=dev)  # device-side: no host copy
    q_off = (two * m).expand(b, 2).contiguous()
    k_off = (two * n).expand(b, 2).contiguous()
    ids = torch.zeros((b, 1, 1), dtype=torch.int32, device=dev)
    cnt = torch.ones((b, 1), dtype=torch.int32, device=dev)
    return block_sparse_attention(q_rows.contiguous(), k, v, q_off, k_off, ids, cnt, _ws_tag="attn_dense")


def repair_apply(base: torch.Tensor, state, alpha: float, rows: torch.Tensor | None = None,
                 dense: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Reduced-rank residual repair + probe overwrite on bf16 [B,N,128] (rank 16)."""
    dev = _cuda(base)
    x_mean, x_scale, y_mean, left, basis = (t.to(torch.float32).contiguous() for t in state)
    b, n, d = base.shape
    r = left.shape[-1]
    if out is None:
        out = torch.empty_like(base)
    m = 0 if rows is None else rows.shape[1]
    rows_i = None if rows is None else rows.to(torch.int32).contiguous()
    dense_b = None if dense is None else dense.to(torch.bfloat16).contiguous()
    _count(1 if m == 0 else 2)
    _lib.call("spr_repair_apply", _p(_contig("base", base)), _p(x_mean), _p(x_scale), _p(y_mean), _p(left), _p(basis),
              b, n, d, r, float(alpha), _p(rows_i), _p(dense_b), m, _p(out), _stream(dev))
    return out


def sym_eig(a: torch.Tensor, max_sweeps: int = 15, top: int | None = None):
    """Batched symmetric eigendecomposition of [B,n,n] (n even <= 128):
    (eigenvalues ascending [B,n], eigenvectors in columns [B,n,n]), fp32.
    ``top``: only the eigenvectors of the ``top`` largest eigenvalues are
    formed (the last ``top`` columns; zeros elsewhere for n = 64, 128)."""
    dev = _cuda(a)
    b, n, n2 = a.shape
    if n != n2:
        raise RuntimeError(f"sym_eig expects square matrices, got {tuple(a.shape)}")
    a = a.to(torch.float32).contiguous()
    evals = torch.empty((b, n), dtype=torch.float32, device=dev)
    evecs = torch.empty((b, n, n), dtype=torch.float32, device=dev)
    _count(1)
    if top is None:
        _lib.call("spr_sym_eig", _p(a), b, n, int(max_sweeps), _p(evals), _p(evecs), _stream(dev))
    else:
        _lib.call("spr_sym_eig_top", _p(a), b, n, int(top), int(max_sweeps), _p(evals), _p(evecs), _stream(dev))
    return evals, evecs


def chol_solve(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Solve A X = B for batched SPD A [B,m,m] and B [B,m,r] (fp32); non-PD A gives non-finite X."""
    dev = _cuda(a, b)
    bt, m, _ = a.shape
    a = a.to(torch.float32).contiguous()
    b = b.to(torch.float32).contiguous()
    x = torch.empty_like(b)
    _count(1)
    _lib.call("spr_chol_solve", _p(a), _p(b), bt, m, b.shape[2], _p(x), _stream(dev))
    return x


def wan_qkv_norm_rope_layout(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_weight: torch.Tensor,
                             k_weight: torch.Tensor, freq_real: torch.Tensor, freq_imag: torch.Tensor, heads: int,
                             epsilon: float):
    """Wan RMSNorm + RoPE + [B,L,C] -> [B,H,L,D] layout for Q/K (V: layout only).

    Same arguments and result as the reference's
    ``sparsepr.kernels.n8_extension.wan_qkv_norm_rope_layout``
    (``n8_ops.cu:357-411``): returns ``(q_out, k_out, v_out)``, each
    ``[B, heads, L, C/heads]`` in the input dtype."""
    dev = _cuda(q, k, v, q_weight, k_weight, freq_real, freq_imag)
    for name, t in (("q", q), ("k", k), ("v", v)):
        _contig(name, t)
    if q.shape != k.shape or q.shape != v.shape or q.dim() != 3:
        raise RuntimeError(f"Wan QKV inputs must have matching [B,L,C] shapes, got {tuple(q.shape)}, "
                           f"{tuple(k.shape)}, {tuple(v.shape)}")
    if not (q.dtype == k.dtype == v.dtype == q_weight.dtype == k_weight.dtype) or q.dtype not in _DT:
        raise RuntimeError("Wan QKV inputs and norm weights must share one of fp32/bf16/fp16")
    if freq_real.dtype != torch.float32 or freq_imag.dtype != torch.float32:
        raise RuntimeError("Wan RoPE frequency tensors must be FP32")
    b, l, c = q.shape
    if heads <= 0 or c % heads:
        raise RuntimeError(f"Wan channels ({c}) must divide num_heads ({heads})")
    hd = c // heads
    if q_weight.numel() != c or k_weight.numel() != c:
        raise RuntimeError("Wan norm weights must contain C elements")
    if tuple(freq_real.shape) != (l, hd // 2) or tuple(freq_imag.shape) != (l, hd // 2):
        raise RuntimeError(f"Wan RoPE frequencies must have shape [L,D/2] = [{l},{hd // 2}]")
    outs = [torch.empty((b, heads, l, hd), dtype=q.dtype, device=dev) for _ in range(3)]
    _count(1)
    _lib.call("spr_wan_qkv_norm_rope_layout", _p(q), _p(k), _p(v), _p(q_weight.contiguous()),
              _p(k_weight.contiguous()), _p(freq_real.contiguous()), _p(freq_imag.contiguous()), _DT[q.dtype], b, l,
              c, heads, float(epsilon), _p(outs[0]), _p(outs[1]), _p(outs[2]), _stream(dev))
    return tuple(outs)


def cholesky_qr(x: torch.Tensor, relative_ridge: float):
    """Cholesky-QR with column normalisation and a relative ridge (warm role
    factors): x [B,n,r] fp32 -> (orthonormalised [B,n,r], failed bool [B])."""
    dev = _cuda(x)
    b, n, r = x.shape
    xc = x.float().contiguous()
    out = torch.empty_like(xc)
    failed = torch.empty(b, dtype=torch.int32, device=dev)
    _count(1)
    _lib.call("spr_cholesky_qr", _p(xc), b, n, r, float(relative_ridge), _p(out), _p(failed), _stream(dev))
    return out, failed.bool()


def ridge_cholesky(a: torch.Tensor, scale: torch.Tensor, relative_ridge: float, fallback_ridge: float = 1e-2):
    """Lower Cholesky factor of a + scale*ridge*I with the reference's fallback
    ridge: a [B,m,m], scale [B] -> (L [B,m,m], failed bool [B])."""
    dev = _cuda(a, scale)
    b, m, _ = a.shape
    ac = a.float().contiguous()
    sc = scale.float().contiguous()
    l = torch.empty_like(ac)
    failed = torch.empty(b, dtype=torch.int32, device=dev)
    _count(1)
    _lib.call("spr_ridge_cholesky", _p(ac), _p(sc), b, m, float(relative_ridge), float(fallback_ridge), _p(l),
              _p(failed), _stream(dev))
    return l, failed.bool()
