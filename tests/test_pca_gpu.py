"""Device PCA start of the PCA-initialised openTSNE entry points
(fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_{double,float},
src/embedding_cuda_impl.cpp:142-183) against the restatement oracle.pca_start
(itself pinned against scikit-learn in tests/test_pca_cpu.py)."""
import ctypes

import numpy as np
import pytest

import oracle as O
from fastembedr_b200 import _lib, api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def data():
    x, _ = S.gaussian_mixture(S.MixtureSpec(n=40_000, dim=50, components=8, seed=3))
    return x


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_pca_start_matches_oracle(data, dtype):
    n, p = data.shape
    x = np.ascontiguousarray(data.astype(dtype).T)  # R column-major
    out = np.zeros((n, 2), np.float32)
    _lib.check(_lib.load().fe_b200_pca_start(ctypes.c_void_p(x.ctypes.data), int(dtype == np.float64), n, p,
                                             out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))),
               "fe_b200_pca_start")
    want = O.pca_start(data.astype(dtype))
    err = np.abs(out - want).max() / 1e-4
    print(f"PCA start ({np.dtype(dtype).name}): max |diff| / sd {err:.2e}")
    assert err < 1e-4


def test_pca_entry_point_runs_from_the_start(data):
    """The _pca_float entry point equals the device-KNN entry point started from
    the oracle's PCA start, after one iteration (the starts agree to 1e-4 of
    their 1e-4 scale; one step at learning rate n/12 keeps them close)."""
    import torch

    n, p = data.shape
    idx, dist = S.exact_knn(data, 30, device="cuda")
    d_idx = torch.from_numpy(np.ascontiguousarray(idx.T)).cuda()
    d_dist = torch.from_numpy(np.ascontiguousarray(dist.T)).cuda()
    xcm = np.ascontiguousarray(data.T)
    L = _lib.load()
    out = np.zeros((n, 2), np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    torch.cuda.synchronize()
    rc = L.fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_float(
        ctypes.c_void_p(d_idx.data_ptr()), ctypes.c_void_p(d_dist.data_ptr()), ctypes.c_void_p(xcm.ctypes.data), p,
        n, 30, 2, 10.0, 1, 0, 12.0, 1.0, 0.0, 1, 0.8, 0.8, 0.01, 5.0, 42, 0, out.ctypes.data_as(fp))
    _lib.check(rc, "pca_float")
    init = O.pca_start(data)
    ref = np.zeros((n, 2), np.float32)
    rc = L.fastembedr_cuda_opentsne_fft_from_device_knn_float(
        ctypes.c_void_p(d_idx.data_ptr()), ctypes.c_void_p(d_dist.data_ptr()), init.ctypes.data_as(fp), 1, n, 30, 2,
        10.0, 1, 0, 12.0, 1.0, 0.0, 1, 0.8, 0.8, 0.01, 5.0, 42, 0, ref.ctypes.data_as(fp))
    _lib.check(rc, "device knn")
    assert np.isfinite(out).all()
    rel = float(np.linalg.norm(out - ref) / np.linalg.norm(ref))
    print(f"one iteration from the device PCA start vs from the oracle's: rel-L2 {rel:.2e}")
    assert rel < 1e-3


def test_pca_entry_point_rejects_bad_dimensions(data):
    import torch

    n = 100
    d_idx = torch.zeros((5, n), dtype=torch.int32, device="cuda")
    d_dist = torch.ones((5, n), dtype=torch.float32, device="cuda")
    x = np.zeros(n, np.float64)
    out = np.zeros((n, 2), np.float32)
    rc = _lib.load().fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_double(
        ctypes.c_void_p(d_idx.data_ptr()), ctypes.c_void_p(d_dist.data_ptr()), ctypes.c_void_p(x.ctypes.data), 1,
        n, 5, 2, 3.0, 1, 0, 12.0, 1.0, 0.0, 1, 0.8, 0.8, 0.01, 5.0, 42, 0,
        out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    assert rc == 1
    assert "PCA" in _lib.last_error()
