"""fastembedr_b200 -- B200-native drop-in for fastEmbedR's CUDA embedding optimizer.

The product is ``libfastembedr_b200.so`` (C ABI: ``include/fastembedr_b200.h``),
hand-written sm_100a CUDA for the openTSNE FFT-grid optimizer and the UMAP
COO edge-SGD optimizer.  This package holds its sources (``csrc/``), the build
step (``build_lib``), a ctypes binding (``_lib``), a Python mirror of the
reference's R-level entry points for this path (``api``) and seeded synthetic
inputs (``synthetic``).
"""
from .api import (  # noqa: F401
    EmbeddingResult,
    TsneSession,
    cuda_available,
    find_ab_params,
    opentsne_knn,
    resolve_index_offset,
    tsne_auto_parameters,
    umap_epochs,
    umap_optimize_coo,
    version,
)
from ._lib import CudaBackendError  # noqa: F401

__all__ = [
    "EmbeddingResult", "TsneSession", "CudaBackendError", "cuda_available", "find_ab_params",
    "opentsne_knn", "resolve_index_offset", "tsne_auto_parameters", "umap_epochs",
    "umap_optimize_coo", "version",
]
