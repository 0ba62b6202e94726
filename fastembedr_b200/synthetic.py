"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The reference benchmarks on MNIST / flow18 / ImageNet embeddings, which are
not available here; Gaussian mixtures with the configured sizes stand in for
them.  Exact Euclidean non-self KNN is computed by brute force: NumPy on the
CPU for small n, this library's exact KNN on a GPU (torch's blocked brute
force stays available as an independent producer).

KNN results are ``(n, k)`` int32 indices (0-based, self excluded, sorted by
distance) and float32 distances; ``column_major`` converts to the R layout the
C ABI takes (``idx[j*n + i]``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np


@dataclass(frozen=True)
class MixtureSpec:
    n: int
    dim: int = 50
    components: int = 10
    mean_sd: float = 4.0          # means ~ N(0, 16 I)
    anisotropic: bool = False     # per-component diagonal sd ~ U(0.5, 2)
    dirichlet_weights: bool = False
    seed: int = 0


# The benchmark configurations (KNN width, perplexity, schedule live with callers).
CONFIGS = {
    "tsne_10k": MixtureSpec(n=10_000, components=10),
    "umap_70k": MixtureSpec(n=70_000, components=10),
    "tsne_70k": MixtureSpec(n=70_000, components=10, anisotropic=True),
    "tsne_1m": MixtureSpec(n=1_000_000, components=20, anisotropic=True, dirichlet_weights=True),
    "umap_2m": MixtureSpec(n=2_000_000, components=20),
    # the north star's scaling size for t-SNE (N >= 2M), generated as tsne_1m
    "tsne_2m": MixtureSpec(n=2_000_000, components=20, anisotropic=True, dirichlet_weights=True),
    # profiling stand-in for tsne_1m: same generator, P (~0.25 GB) still larger than L2
    "tsne_200k": MixtureSpec(n=200_000, components=20, anisotropic=True, dirichlet_weights=True),
}


def gaussian_mixture(spec: MixtureSpec) -> Tuple[np.ndarray, np.ndarray]:
    """Points (n, dim) float32 and component labels (n,) int32."""
    rng = np.random.default_rng(spec.seed)
    means = rng.normal(0.0, spec.mean_sd, size=(spec.components, spec.dim))
    if spec.anisotropic:
        sds = rng.uniform(0.5, 2.0, size=(spec.components, spec.dim))
    else:
        sds = np.ones((spec.components, spec.dim))
    if spec.dirichlet_weights:
        weights = rng.dirichlet(np.ones(spec.components))
        labels = rng.choice(spec.components, size=spec.n, p=weights)
    else:
        labels = np.arange(spec.n) % spec.components
        rng.shuffle(labels)
    x = rng.standard_normal(size=(spec.n, spec.dim)) * sds[labels] + means[labels]
    return x.astype(np.float32), labels.astype(np.int32)


def exact_knn_numpy(x: np.ndarray, k: int, block: int = 1024) -> Tuple[np.ndarray, np.ndarray]:
    n = x.shape[0]
    xd = x.astype(np.float64)
    sq = np.einsum("ij,ij->i", xd, xd)
    idx = np.empty((n, k), np.int32)
    dist = np.empty((n, k), np.float32)
    for s in range(0, n, block):
        e = min(n, s + block)
        d2 = sq[s:e, None] - 2.0 * xd[s:e] @ xd.T + sq[None, :]
        d2[np.arange(e - s), np.arange(s, e)] = np.inf
        part = np.argpartition(d2, k, axis=1)[:, :k]
        pd = np.take_along_axis(d2, part, axis=1)
        order = np.lexsort((part, pd), axis=1)
        sel = np.take_along_axis(part, order, axis=1)
        idx[s:e] = sel
        diff = x[s:e, None, :].astype(np.float64) - x[sel].astype(np.float64)
        dist[s:e] = np.sqrt(np.einsum("ijk,ijk->ij", diff, diff)).astype(np.float32)
    return idx, dist


def exact_knn_torch(x: np.ndarray, k: int, device: str = "cuda",
                    block: int = 2048) -> Tuple[np.ndarray, np.ndarray]:
    """Blocked brute force on a GPU: fp32 distance GEMM, top-(k+1), exact re-evaluation."""
    import torch

    with torch.no_grad():
        prev_tf32 = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        X = torch.from_numpy(x).to(device)
        sq = (X * X).sum(1)
        n = X.shape[0]
        idx = torch.empty((n, k), dtype=torch.int32, device=device)
        dist = torch.empty((n, k), dtype=torch.float32, device=device)
        for s in range(0, n, block):
            e = min(n, s + block)
            d2 = sq[s:e, None] - 2.0 * (X[s:e] @ X.T) + sq[None, :]
            d2[torch.arange(e - s, device=device), torch.arange(s, e, device=device)] = float("inf")
            _, sel = torch.topk(d2, k, dim=1, largest=False, sorted=True)
            diff = X[s:e, None, :] - X[sel]
            dd = torch.sqrt((diff.double() ** 2).sum(-1)).float()
            dd, order = torch.sort(dd, dim=1, stable=True)
            idx[s:e] = torch.gather(sel, 1, order).int()
            dist[s:e] = dd
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32
        return idx.cpu().numpy(), dist.cpu().numpy()


def exact_knn(x: np.ndarray, k: int, device: Optional[str] = None, producer: str = "b200") -> Tuple[np.ndarray, np.ndarray]:
    """Exact non-self KNN: on a GPU with this library's producer
    (fe_b200_knn_exact) by default, or torch's blocked brute force
    (producer="torch", an independent implementation); NumPy without a device."""
    if device is not None and device.startswith("cuda"):
        if producer == "b200":
            import torch

            from . import api

            with torch.cuda.device(torch.device(device)):
                return api.knn_exact(x, k)
        return exact_knn_torch(x, k, device)
    return exact_knn_numpy(x, k)


def column_major(a: np.ndarray) -> np.ndarray:
    """(n, k) -> contiguous R column-major buffer (length n*k)."""
    return np.ascontiguousarray(a.T).reshape(-1)


def tsne_init(n: int, seed: int = 0) -> np.ndarray:
    """R's default openTSNE init: N(0, 1e-4^2), centred (R/tsne_control.R:285-292, 331-335)."""
    rng = np.random.default_rng(seed)
    y = rng.normal(0.0, 1e-4, size=(n, 2)).astype(np.float32)
    return (y - y.mean(0, dtype=np.float64).astype(np.float32)).astype(np.float32)


def umap_random_init(n: int, seed: int = 0, scale: float = 10.0) -> np.ndarray:
    """Spectral-free random init U(-scale, scale)."""
    rng = np.random.default_rng(seed)
    return rng.uniform(-scale, scale, size=(n, 2)).astype(np.float32)
