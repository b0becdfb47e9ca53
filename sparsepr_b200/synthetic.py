"""Seeded synthetic inputs with the shapes and statistics of the benchmark configs.

There is no public dataset for this path; the inputs are fully defined by the
configuration: Q and K are 3D-smooth Gaussian random fields over the latent
(t, h, w) grid plus white noise, V is white noise, and the standalone k-means
points are a smooth mixture of Gaussians.  Used by the tests, ``bench.py``
and ``__graft_entry__.smoke()``.
"""

from __future__ import annotations

import torch

__all__ = [
    "gaussian_blur_matrix",
    "smooth_field",
    "synthetic_qkv",
    "synthetic_qkv_heads",
    "synthetic_kmeans_points",
    "kmeans_plus_plus",
    "random_init_indices",
]


def gaussian_blur_matrix(n: int, sigma: float, device=None) -> torch.Tensor:
    """Row-normalised Gaussian kernel truncated at the grid edge, [n, n] fp32."""
    i = torch.arange(n, device=device, dtype=torch.float32)
    g = torch.exp(-((i[:, None] - i[None, :]) ** 2) / (2.0 * sigma * sigma))
    return g / g.sum(dim=1, keepdim=True)


def smooth_field(channels: int, grid: tuple[int, int, int], sigma: float,
                 generator: torch.Generator, device=None) -> torch.Tensor:
    """``channels`` independent unit-variance smooth fields -> [channels, T*H*W] fp32."""
    t, h, w = grid
    x = torch.randn((channels, t, h, w), generator=generator, device=device, dtype=torch.float32)
    for axis, n in ((1, t), (2, h), (3, w)):
        g = gaussian_blur_matrix(n, sigma, device=device)
        x = torch.movedim(torch.tensordot(x, g, dims=([axis], [1])), -1, axis)
    x = x.reshape(channels, -1)
    x = (x - x.mean(dim=1, keepdim=True)) / x.std(dim=1, keepdim=True).clamp_min(1e-12)
    return x


def synthetic_qkv(heads: int, head_dim: int, grid: tuple[int, int, int], *, batch: int = 1,
                  sigma: float = 2.0, noise: float = 0.5, dtype=torch.bfloat16,
                  device=None, seeds=(0, 1, 2)):
    """Q, K as smooth field + ``noise``·N(0,1), V ~ N(0,1); each [B,H,N,D] in ``dtype``.

    Q, K, V use ``torch.Generator`` seeds ``seeds[0..2]`` on ``device``.
    """
    n = grid[0] * grid[1] * grid[2]
    out = []
    for role, seed in zip("qkv", seeds):
        g = torch.Generator(device=device if device is not None else "cpu").manual_seed(int(seed))
        if role == "v":
            x = torch.randn((batch * heads * head_dim, n), generator=g, device=device)
        else:
            x = smooth_field(batch * heads * head_dim, grid, sigma, g, device=device)
            x = x + noise * torch.randn(x.shape, generator=g, device=device)
        x = x.view(batch, heads, head_dim, n).transpose(2, 3).contiguous()
        out.append(x.to(dtype))
    return tuple(out)


def synthetic_qkv_heads(h0: int, h1: int, head_dim: int, grid: tuple[int, int, int], *, sigma: float = 2.0,
                        noise: float = 0.5, dtype=torch.bfloat16, device=None, seeds=(0, 1, 2)):
    """Heads ``[h0, h1)`` of a per-head-seeded Q/K/V set, each [1, h1-h0, N, D].

    Head ``h`` of role ``r`` draws from its own generator (seed
    ``seeds[r] * 1_000_003 + h``), so any head range (one rank's shard, a CPU
    sample) equals the same heads of the full set, whatever the sharding.
    Same statistics as :func:`synthetic_qkv`.
    """
    n = grid[0] * grid[1] * grid[2]
    out = []
    for role, seed in zip("qkv", seeds):
        t = torch.empty((1, h1 - h0, n, head_dim), dtype=dtype, device=device)
        for i, h in enumerate(range(h0, h1)):
            g = torch.Generator(device=device if device is not None else "cpu").manual_seed(
                int(seed) * 1_000_003 + int(h))
            if role == "v":
                x = torch.randn((head_dim, n), generator=g, device=device)
            else:
                x = smooth_field(head_dim, grid, sigma, g, device=device)
                x = x + noise * torch.randn(x.shape, generator=g, device=device)
            t[0, i] = x.t().to(dtype)
        out.append(t)
    return tuple(out)


def synthetic_kmeans_points(problems: int, dim: int, grid: tuple[int, int, int], components: int, *,
                            sigma: float = 2.0, noise: float = 0.3, dtype=torch.bfloat16,
                            device=None, seed: int = 0) -> torch.Tensor:
    """Mixture of ``components`` Gaussians whose component map is smooth over the grid.

    Component means ~ 2·N(0, I); each token takes the argmax over
    ``components`` smooth fields; point = mean + ``noise``·N(0,1).
    Returns [problems, T*H*W, dim].
    """
    g = torch.Generator(device=device if device is not None else "cpu").manual_seed(int(seed))
    n = grid[0] * grid[1] * grid[2]
    out = torch.empty((problems, n, dim), dtype=dtype, device=device)
    for p in range(problems):
        means = 2.0 * torch.randn((components, dim), generator=g, device=device)
        comp = smooth_field(components, grid, sigma, g, device=device).argmax(dim=0)
        pts = means[comp] + noise * torch.randn((n, dim), generator=g, device=device)
        out[p] = pts.to(dtype)
    return out


def random_init_indices(bh: int, n: int, k: int, seed: int) -> torch.Tensor:
    """Seeded random-sample initial centroid indices ``randint(0, N, (BH, K))``,
    the reference's cold-start rule (``flash_kmeans/kmeans_triton_impl.py:89-96``),
    drawn on a CPU generator so the indices do not depend on the device."""
    g = torch.Generator().manual_seed(int(seed))
    return torch.randint(0, n, (bh, k), generator=g)


def kmeans_plus_plus(x: torch.Tensor, k: int, seed: int) -> torch.Tensor:
    """Seeded k-means++ seeding per problem: x [B,N,D] -> centroids [B,K,D] fp32.

    D² sampling with float64 distances on x's device; the uniform draws come
    from a CPU generator so CPU and GPU runs pick the same points whenever
    their distances agree.
    """
    b, n, d = x.shape
    g = torch.Generator().manual_seed(int(seed))
    xf = x.double()
    ar = torch.arange(b, device=x.device)
    first = torch.randint(0, n, (b,), generator=g).to(x.device)
    idx = torch.empty((b, k), dtype=torch.long, device=x.device)
    idx[:, 0] = first
    dmin = (xf - xf[ar, first][:, None]).square().sum(-1)
    for j in range(1, k):
        u = torch.rand((b,), generator=g, dtype=torch.float64).to(x.device)
        cdf = dmin.cumsum(dim=1)
        pick = torch.searchsorted(cdf, (u * cdf[:, -1]).unsqueeze(1)).squeeze(1).clamp_max(n - 1)
        idx[:, j] = pick
        dmin = torch.minimum(dmin, (xf - xf[ar, pick][:, None]).square().sum(-1))
    return torch.gather(x.float(), 1, idx.unsqueeze(-1).expand(-1, -1, d))
