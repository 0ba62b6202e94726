"""Generate umap_device_small.npz from the reference's own CUDA backend.

The device-KNN UMAP path of the reference (src/embedding_cuda_kernels.cpp)
exists only as CUDA code, so its golden vectors come from that file compiled
unmodified into ``oracle/_ref/libferef_cuda.so`` (``oracle/Makefile``) and run
on a GPU.  Run from the repository root on a machine with a GPU:

    python tests/golden/make_golden_cuda.py [--out DIR]

Inputs (stored in the fixture):
  lowd_*  -- 2-D Gaussian mixture, n = 1000, exact k = 15 KNN.  No row of its
             fuzzy graph reaches the reference's row capacity (2k = 30), so
             the reference's graph is fully determined.
  hub_*   -- the 50-D KNN of umap_small.npz, where hub vertices overflow their
             rows and the reference keeps an arbitrary subset of incoming edges.
Outputs: the reference's graph dumps (rank-major COO) for both, and for lowd
the fused path's layout after 1 epoch (the diffusion start, sanitised) in
fuzzy and binary graph modes and after 3 epochs in the Jacobi (delta) mode.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402
from fastembedr_b200 import synthetic as S  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
SEED, SPECTRAL_ITERS = 42, 30
A, B = 1.5769434601962196, 0.8950608781227859


def lowd_knn():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(c, 1.0, (250, 2)) for c in rng.normal(0, 6, (4, 2))]).astype(np.float32)
    return S.exact_knn_numpy(x, 15)


def ref_device_binary_start(idx, dist):
    """fastembedr_cuda_umap_from_device_knn_spectral_float with binary_graph = 1, one epoch."""
    import torch

    C = O.ref_cuda()
    fn = C.fastembedr_cuda_umap_from_device_knn_spectral_float
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 4 + [ctypes.c_float] * 4 + [
        ctypes.c_int, ctypes.c_uint, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    n, k = idx.shape
    d_idx = torch.from_numpy(np.ascontiguousarray(idx.T)).cuda()
    d_dist = torch.from_numpy(np.ascontiguousarray(dist.T)).cuda()
    out = np.zeros((n, 2), np.float32)
    rc = fn(d_idx.data_ptr(), d_dist.data_ptr(), n, k, 1, 5, 1.0, A, B, 1.0, SPECTRAL_ITERS, SEED, 0, 1, 1,
            out.ctypes.data)
    O._ref_cuda_check(rc, "fused UMAP (device, binary)")
    return out


def main():
    out_dir = sys.argv[sys.argv.index("--out") + 1] if "--out" in sys.argv else OUT
    lidx, ldist = lowd_knn()
    small = np.load(os.path.join(OUT, "umap_small.npz"))
    hidx, hdist = small["idx"], small["dist"]
    ld = O.ref_cuda_umap_graph_dump(lidx, ldist)
    hd = O.ref_cuda_umap_graph_dump(hidx, hdist)
    start = O.ref_cuda_umap_fused(lidx, ldist, n_epochs=1, spectral_n_iter=SPECTRAL_ITERS, seed=SEED)
    start_binary = ref_device_binary_start(lidx, ldist)
    delta3 = O.ref_cuda_umap_fused(lidx, ldist, n_epochs=3, spectral_n_iter=SPECTRAL_ITERS, seed=SEED,
                                   optimizer_mode=1)
    np.savez_compressed(
        os.path.join(out_dir, "umap_device_small.npz"),
        lowd_idx=lidx, lowd_dist=ldist,
        lowd_heads=ld["heads"], lowd_tails=ld["tails"], lowd_weights=ld["weights"],
        lowd_epochs_per_sample=ld["epochs_per_sample"], lowd_width=ld["width"],
        hub_heads=hd["heads"], hub_tails=hd["tails"], hub_weights=hd["weights"],
        hub_epochs_per_sample=hd["epochs_per_sample"],
        lowd_start=start, lowd_start_binary=start_binary, lowd_delta3=delta3,
        seed=SEED, spectral_n_iter=SPECTRAL_ITERS)
    print("wrote umap_device_small.npz:", ld["capacity"], "lowd edges,", hd["capacity"], "hub edges")


if __name__ == "__main__":
    main()
