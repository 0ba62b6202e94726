"""The allocation-free UMAP entry point against the allocating one.

fe_b200_umap_epochs_noalloc exists for callers that cannot let a library
allocate device memory (frameworks that own the device heap through their own
allocator, real-time loops where cudaMalloc/cudaFree would synchronise the
device, fixed memory budgets).  It runs on caller-owned device buffers and
keeps its only scratch in a fixed static device array.  This file checks, on
two calls in a row, that it produces what fe_b200_umap_epochs (the allocating
entry point, Jacobi mode) produces for the same inputs, within the 1e-4
absolute tolerance the UMAP parity tests hold each epoch to, and that the second call leaves
the device's free memory unchanged.  It is named to run after every other test
file and passes on its own as well.
"""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

A, B = 1.5769434601962196, 0.8950608781227859
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "umap_small.npz")


def _noalloc(lib, d_heads, d_tails, d_eps, d_layout, n, e0, e1, n_epochs, stream=None):
    return lib.fe_b200_umap_epochs_noalloc(
        ctypes.c_void_p(d_heads.data_ptr()), ctypes.c_void_p(d_tails.data_ptr()),
        ctypes.c_void_p(d_eps.data_ptr()), d_heads.numel(), ctypes.c_void_p(d_layout.data_ptr()), n, e0, e1,
        n_epochs, 5, 1.0, A, B, 1.0, 42, 0, stream)


def test_no_alloc_entry_point_matches_allocating_one():
    import torch

    from fastembedr_b200 import _lib, api

    g = np.load(GOLDEN)
    heads = np.repeat(np.arange(g["offsets"].size - 1), np.diff(g["offsets"])).astype(np.int32)
    tails = g["neighbors"].astype(np.int32)
    eps = g["epochs_per_sample"].astype(np.float32)
    y0 = g["init"].astype(np.float32)
    n = y0.shape[0]
    lib = _lib.load()

    d_heads = torch.from_numpy(heads).cuda()
    d_tails = torch.from_numpy(tails).cuda()
    d_eps = torch.from_numpy(eps).cuda()
    d_layout = torch.from_numpy(y0.copy()).cuda()
    torch.cuda.synchronize()

    # Two calls in a row, one epoch each; the second continues from the first
    # call's layout, and the allocating entry point starts from that same layout
    # (the 1e-4 bar is per epoch: float atomics order the delta sums freely).
    for call, (e0, e1) in enumerate(((1, 2), (2, 3))):
        start = d_layout.cpu().numpy()
        want, _ = api.umap_epochs(heads, tails, eps, start, e0, e1, 10, a=A, b=B, optimizer_mode=1)
        free_before = torch.cuda.mem_get_info()[0]
        rc = _noalloc(lib, d_heads, d_tails, d_eps, d_layout, n, e0, e1, 10)
        assert rc == 0, _lib.last_error()
        if call == 1:  # the first call on the device loads the library's static scratch
            assert torch.cuda.mem_get_info()[0] == free_before
        got = d_layout.cpu().numpy()
        assert np.isfinite(got).all()
        assert np.abs(got - want).max() < 1e-4


def test_no_alloc_entry_point_rejects_oversized_graphs():
    import torch

    from fastembedr_b200 import _lib

    lib = _lib.load()
    d = torch.zeros(4, dtype=torch.int32, device="cuda")
    f = torch.zeros(4, dtype=torch.float32, device="cuda")
    rc = lib.fe_b200_umap_epochs_noalloc(
        ctypes.c_void_p(d.data_ptr()), ctypes.c_void_p(d.data_ptr()), ctypes.c_void_p(f.data_ptr()), 4,
        ctypes.c_void_p(f.data_ptr()), (1 << 20) + 1, 0, 1, 10, 5, 1.0, A, B, 1.0, 42, 0, None)
    assert rc == 1
    assert "exceeds the fixed scratch capacity" in _lib.last_error()
