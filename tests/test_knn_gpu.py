"""Exact KNN on the B200 (fe_b200_knn_exact, the GPU-KNN producer) against an
independent exact KNN: NumPy in double (synthetic.exact_knn_numpy) at small n
and the torch brute force with double re-evaluation at larger n.

Bars: the same neighbour sets, position by position, except where two
candidates lie within float rounding of each other (then at most a swap);
distances within 1e-6 relative; the reference's GPU-KNN layout (column-major
n x k, 1-based, self excluded)."""
import time

import numpy as np
import pytest

from fastembedr_b200 import api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu


def _compare(idx, dist, ridx, rdist, rtol=1e-6):
    assert idx.shape == ridx.shape and dist.shape == rdist.shape
    same = idx == ridx
    frac = float(same.mean())
    # any mismatch must be a near-tie: the two distances agree to float rounding
    bad = ~same
    np.testing.assert_allclose(dist[bad], rdist[bad], rtol=1e-5)
    np.testing.assert_allclose(dist, rdist, rtol=rtol, atol=1e-6)
    return frac


@pytest.mark.parametrize("n,p,k", [(3001, 50, 90), (2500, 100, 15), (777, 7, 30)])
def test_knn_matches_numpy_exact(n, p, k):
    x, _ = S.gaussian_mixture(S.MixtureSpec(n=n, dim=p, components=6, seed=n))
    idx, dist = api.knn_exact(x, k)
    # row-major (n, k), as every KNN of this package (torch.distributed
    # broadcasts and the column-major helpers need contiguous arrays)
    assert idx.flags.c_contiguous and dist.flags.c_contiguous
    ridx, rdist = S.exact_knn_numpy(x, k)
    frac = _compare(idx, dist, ridx, rdist)
    print(f"n={n} p={p} k={k}: {frac:.6f} of entries identical")
    assert frac > 0.999
    assert not (idx == np.arange(n)[:, None]).any()  # self excluded


def test_knn_matches_torch_at_scale():
    x, _ = S.gaussian_mixture(S.MixtureSpec(n=60_000, dim=50, components=10, seed=2, anisotropic=True))
    t0 = time.perf_counter()
    idx, dist = api.knn_exact(x, 90)
    t1 = time.perf_counter()
    ridx, rdist = S.exact_knn_torch(x, 90)
    t2 = time.perf_counter()
    # torch's re-evaluation forms q - x in float before squaring in double;
    # this library (and NumPy) difference in double: a few ulps apart.
    frac = _compare(idx, dist, ridx, rdist, rtol=1e-5)
    print(f"n=60k k=90: {frac:.6f} identical; ours {t1 - t0:.2f}s, torch {t2 - t1:.2f}s")
    assert frac > 0.999


def test_knn_device_layout_and_double_input():
    import torch

    x, _ = S.gaussian_mixture(S.MixtureSpec(n=1500, dim=20, components=4, seed=9))
    d_idx, d_dist = api.knn_exact(torch.from_numpy(x.astype(np.float64)).cuda(), 12, device_output=True)
    assert d_idx.shape == (12, 1500) and d_idx.dtype == torch.int32 and d_idx.is_cuda
    idx = d_idx.t().cpu().numpy()
    assert idx.min() >= 1 and idx.max() <= 1500  # 1-based
    ridx, rdist = S.exact_knn_numpy(x, 12)
    assert float((idx - 1 == ridx).mean()) > 0.999
    np.testing.assert_allclose(d_dist.t().cpu().numpy(), rdist, rtol=1e-6, atol=1e-6)


def test_knn_feeds_the_device_knn_entry_point():
    """The producer's output goes straight into the device-KNN openTSNE entry
    point (index_offset 1), as the reference's GPU-KNN object does."""
    x, _ = S.gaussian_mixture(S.MixtureSpec(n=4000, dim=30, components=5, seed=4))
    d_idx, d_dist = api.knn_exact(x, 45, device_output=True)
    idx, dist = api.knn_exact(x, 45)
    a = api.opentsne_knn(d_idx.t(), d_dist.t(), perplexity=15.0, n_iter=50, early_exaggeration_iter=50,
                         index_offset=1).Y
    b = api.opentsne_knn(idx, dist, perplexity=15.0, n_iter=50, early_exaggeration_iter=50).Y
    assert np.array_equal(a, b)


def test_knn_rejects_bad_k():
    x = np.zeros((10, 3), np.float32)
    with pytest.raises(api.CudaBackendError, match="k in"):
        api.knn_exact(x, 10)
