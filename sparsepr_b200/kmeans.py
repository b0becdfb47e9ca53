"""Standalone batched Euclidean k-means on the B200 kernels.

Drop-in for ``src/sparsepr/kmeans_utils.py:1504-1580`` ``batch_kmeans_Euclid``
and ``src/flash_kmeans/interface.py:27-287`` ``FlashKMeans`` (Euclidean,
in-GPU-memory path).  The whole Lloyd loop, including the ``tol`` stop, runs
on the device without host synchronisation.
"""

from __future__ import annotations

import torch

from . import kernels as K
from .synthetic import random_init_indices

__all__ = ["batch_kmeans_Euclid", "FlashKMeans"]


def batch_kmeans_Euclid(x, n_clusters, max_iters=100, tol=1e-4, init_centroids=None, verbose=False,
                        backend="b200", *, seed: int = 0, round_centroids_to_input: bool = False,
                        precision: str = "tf32"):
    """Batched Lloyd k-means.

    Returns ``(cluster_ids int32 [B,N], centroids fp32 [B,K,D], cluster_sizes
    int32 [B,K], n_iters)`` like the reference (which returns int64 ids/sizes
    and a host int); ``n_iters`` here is a 1-element device tensor so the
    call never synchronises.  ``init_centroids=None`` samples
    ``randint(0, N, (B, K))`` rows from a CPU generator seeded by ``seed``
    (the reference draws from the global RNG, ``kmeans_triton_impl.py:89-96``).
    ``round_centroids_to_input`` reproduces the standalone flash_kmeans path,
    which keeps centroids in the input dtype between iterations.
    """
    del verbose, backend
    if max_iters < 0:
        raise RuntimeError(f"max_iters must be non-negative, got {max_iters}.")
    if x.ndim != 3:
        raise RuntimeError(f"Batched k-means expects [B, N, D] input, got shape {tuple(x.shape)}.")
    b, n, d = x.shape
    if init_centroids is None:
        idx = random_init_indices(b, n, n_clusters, seed).to(x.device)
        init_centroids = torch.gather(x, 1, idx.unsqueeze(-1).expand(-1, -1, d))
    init = init_centroids.reshape(b, n_clusters, d).float()
    if max_iters == 0:
        labels = K.kmeans_assign(x.contiguous(), init.contiguous(), precision)
        sizes, _off, _ord = K.label_sort(labels, n_clusters)
        return labels, init, sizes, torch.zeros(1, dtype=torch.int32, device=x.device)
    labels, cent, sizes, _off, _order, iters = K.kmeans_lloyd(
        x.contiguous(), init, max_iters, tol, round_centroids_to_input=round_centroids_to_input, precision=precision)
    return labels, cent, sizes, iters


class FlashKMeans:
    """sklearn-like batched k-means (``flash_kmeans/interface.py:27-287``), CUDA inputs only."""

    def __init__(self, d: int, k: int, niter: int = 25, tol: float = 1e-8, seed: int = 0,
                 verbose: bool = False, dtype: torch.dtype | None = None, device: torch.device | None = None, **_):
        self.d, self.k, self.niter, self.tol, self.seed = int(d), int(k), int(niter), float(tol), int(seed)
        self.verbose = bool(verbose)
        self.dtype = dtype
        self.device = device if device is not None else torch.device("cuda:0")
        self.centroids_b = None
        self.cluster_ids_b = None
        self._batch_size = None

    @staticmethod
    def _batched(data: torch.Tensor):
        if data.ndim == 2:
            return None, data.unsqueeze(0)
        if data.ndim == 3:
            return data.shape[0], data
        raise ValueError("data must be of shape (n_samples, n_features) or (batch_size, n_samples, n_features)")

    def train(self, data: torch.Tensor):
        bsz, x = self._batched(data)
        x = x.to(device=self.device, dtype=self.dtype or x.dtype)
        ids, cents, _sizes, _it = batch_kmeans_Euclid(
            x, self.k, max_iters=self.niter, tol=self.tol, seed=self.seed, round_centroids_to_input=True)
        self.centroids_b = cents
        self.cluster_ids_b = ids
        self._batch_size = bsz

    def fit(self, data: torch.Tensor):
        self.train(data)
        return self

    def predict(self, data: torch.Tensor) -> torch.Tensor:
        if self.centroids_b is None:
            raise RuntimeError("Model not trained. Call train() or fit() first.")
        bsz, x = self._batched(data)
        if bsz != self._batch_size:
            raise ValueError(
                f"Model was trained with batch size B={self._batch_size}, but predict received B={bsz}. "
                "Provide matching batch size."
            )
        x = x.to(device=self.device, dtype=self.dtype or x.dtype).contiguous()
        labels = K.kmeans_assign(x, self.centroids_b.contiguous())
        return labels.squeeze(0) if bsz is None else labels

    def fit_predict(self, data: torch.Tensor) -> torch.Tensor:
        self.train(data)
        return self.cluster_ids_b.squeeze(0) if self._batch_size is None else self.cluster_ids_b
