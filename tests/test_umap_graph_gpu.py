"""The device-KNN UMAP path on the B200 (fuzzy graph, diffusion start, fused
epochs) through the C ABI, against the oracle restatement and against golden
vectors of the reference's own CUDA backend (tests/golden/umap_device_small.npz).

Bars: graph structure identical (heads and tails, index work); graph weights
within 1e-5 relative of the reference's (both use CUDA's expf) and 1e-4 of the
C restatement's (the C library's expf differs in the last bits, which can move
a row's bandwidth bisection by up to its 1e-5 stopping band); start layout
within 1e-6 absolute of the oracle (values are O(1/sqrt(n))) and 1e-5 of the
reference (whose slot order, hence summation order, varies); one Jacobi epoch
on the identical edge schedule within 1e-4 absolute; end-to-end quality within
2% of the reference's own fused path.

The epoch checks feed the oracle the library's own edge list: the schedule
floor(e / p) - floor((e - 1) / p) with p = 1 / w is discontinuous in w, so
weights that differ in the fifth digit can change which edges fire.
"""
import ctypes
import os

import numpy as np
import pytest

import oracle as O
from fastembedr_b200 import _lib, api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu

A, B = 1.5769434601962196, 0.8950608781227859
HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "umap_device_small.npz")


@pytest.fixture(scope="module")
def dev_golden():
    if not os.path.exists(FIXTURE):
        pytest.skip("umap_device_small.npz not generated (tests/golden/make_golden_cuda.py)")
    return np.load(FIXTURE)


@pytest.fixture(scope="module")
def hub_knn(umap_golden):
    return umap_golden["idx"], umap_golden["dist"]


def _rows(heads, tails, weights, n):
    order = np.lexsort((tails, heads))
    h, t, w = heads[order], tails[order], weights[order]
    bounds = np.searchsorted(h, np.arange(n + 1))
    return [(t[bounds[i]:bounds[i + 1]], w[bounds[i]:bounds[i + 1]]) for i in range(n)]


def _oracle_coo(idx, dist, rank_major=True, binary=False):
    nbr, w = O.umap_device_graph(idx, dist, binary=binary)
    return nbr, w, O.umap_pack_coo(nbr, w, rank_major)


@pytest.mark.parametrize("which", ["lowd", "hub"])
def test_graph_dump_matches_oracle(dev_golden, hub_knn, which):
    idx, dist = (dev_golden["lowd_idx"], dev_golden["lowd_dist"]) if which == "lowd" else hub_knn
    got = api.umap_graph_dump(idx, dist)
    _, _, want = _oracle_coo(idx, dist)
    assert got["width"] == 2 * idx.shape[1]
    np.testing.assert_array_equal(got["heads"], want["heads"])
    np.testing.assert_array_equal(got["tails"], want["tails"])
    np.testing.assert_allclose(got["weights"], want["weights"], rtol=1e-4)
    np.testing.assert_allclose(got["epochs_per_sample"], want["epochs_per_sample"], rtol=1e-4)


def test_graph_dump_matches_reference_cuda(dev_golden, hub_knn):
    """Row by row against the reference's dump: every row of the low-dimensional
    graph; in the hub graph, rows below capacity exactly, full rows by size and
    by their own KNN entries."""
    idx, dist = dev_golden["lowd_idx"], dev_golden["lowd_dist"]
    n = idx.shape[0]
    got = api.umap_graph_dump(idx, dist)
    ours = _rows(got["heads"], got["tails"], got["weights"], n)
    ref = _rows(dev_golden["lowd_heads"], dev_golden["lowd_tails"], dev_golden["lowd_weights"], n)
    for (t, w), (tr, wr) in zip(ours, ref):
        np.testing.assert_array_equal(t, tr)
        np.testing.assert_allclose(w, wr, rtol=1e-5)

    idx, dist = hub_knn
    n, width = idx.shape[0], 2 * idx.shape[1]
    got = api.umap_graph_dump(idx, dist)
    ours = _rows(got["heads"], got["tails"], got["weights"], n)
    ref = _rows(dev_golden["hub_heads"], dev_golden["hub_tails"], dev_golden["hub_weights"], n)
    full = 0
    for i, ((t, w), (tr, wr)) in enumerate(zip(ours, ref)):
        if tr.size < width:
            np.testing.assert_array_equal(t, tr)
            np.testing.assert_allclose(w, wr, rtol=1e-5)
        else:
            full += 1
            assert t.size == width
            own = np.unique(idx[i][idx[i] != i])
            assert np.isin(own, t).all() and np.isin(own, tr).all()
    assert full > 0  # the hub graph does exercise the capacity rule


def test_start_layout_matches_oracle(dev_golden):
    idx, dist = dev_golden["lowd_idx"], dev_golden["lowd_dist"]
    y = api.umap_knn(idx, dist, n_epochs=1, spectral_n_iter=30, seed=42).Y
    nbr, w, _ = _oracle_coo(idx, dist)
    want = O.umap_diffusion_init(nbr, w, 42, 30)
    np.testing.assert_allclose(y, want, atol=1e-6)
    # whitened: centred, unit column norms
    np.testing.assert_allclose(y.mean(0), 0.0, atol=1e-6)
    np.testing.assert_allclose((y.astype(np.float64) ** 2).sum(0), 1.0, rtol=1e-4)


def test_start_layout_matches_reference_cuda(dev_golden):
    idx, dist = dev_golden["lowd_idx"], dev_golden["lowd_dist"]
    y = api.umap_knn(idx, dist, n_epochs=1, spectral_n_iter=30, seed=42).Y
    np.testing.assert_allclose(y, dev_golden["lowd_start"], atol=1e-5)


def test_binary_graph_start_layout(dev_golden):
    import torch

    idx, dist = dev_golden["lowd_idx"], dev_golden["lowd_dist"]
    y = api.umap_knn(torch.from_numpy(idx).cuda(), torch.from_numpy(dist).cuda(), n_epochs=1, spectral_n_iter=30,
                     seed=42, graph_mode="binary").Y
    nbr, w, _ = _oracle_coo(idx, dist, binary=True)
    np.testing.assert_allclose(y, O.umap_diffusion_init(nbr, w, 42, 30), atol=1e-6)
    np.testing.assert_allclose(y, dev_golden["lowd_start_binary"], atol=1e-5)


def test_fused_delta_epoch_matches_oracle(dev_golden):
    """n_epochs = 2: epoch 0 applies nothing, epoch 1 is one Jacobi epoch from the
    diffusion start over the library's own edge list."""
    idx, dist = dev_golden["lowd_idx"], dev_golden["lowd_dist"]
    y = api.umap_knn(idx, dist, n_epochs=2, spectral_n_iter=30, seed=42, min_dist=0.1, optimizer_mode=1).Y
    start = api.umap_knn(idx, dist, n_epochs=1, spectral_n_iter=30, seed=42).Y
    coo = api.umap_graph_dump(idx, dist)
    want = O.umap_epoch_delta(coo["heads"], coo["tails"], coo["epochs_per_sample"], start, 1, 2, a=A, b=B,
                              seed=42, hash_key_is_tail=True)
    np.testing.assert_allclose(y, want, atol=1e-4)


def test_fused_delta_epochs_match_reference_cuda(dev_golden):
    """Three epochs (two of them moving) against the reference's fused Jacobi run.
    Both sum each vertex's moves with float atomics in an arbitrary order, and
    the second epoch starts from the first's rounding, hence 1e-3."""
    idx, dist = dev_golden["lowd_idx"], dev_golden["lowd_dist"]
    y = api.umap_knn(idx, dist, n_epochs=3, spectral_n_iter=30, seed=42, min_dist=0.1, optimizer_mode=1).Y
    np.testing.assert_allclose(y, dev_golden["lowd_delta3"], atol=1e-3)


def test_entry_points_agree(dev_golden):
    """Host double, host float and device KNN give the same Jacobi epochs."""
    import torch

    idx, dist = dev_golden["lowd_idx"], dev_golden["lowd_dist"]
    n, k = idx.shape
    kw = dict(n_epochs=3, spectral_n_iter=30, seed=42, min_dist=0.1, optimizer_mode=1)
    y_float = api.umap_knn(idx, dist, **kw).Y
    y_dev = api.umap_knn(torch.from_numpy(idx).cuda(), torch.from_numpy(dist).cuda(), **kw).Y
    idx_cm = np.ascontiguousarray(idx.T)
    dist_cm = np.ascontiguousarray(dist.T.astype(np.float64))
    y_double = np.zeros((n, 2), np.float32)
    rc = _lib.load().fastembedr_cuda_umap_from_knn_spectral(
        ctypes.c_void_p(idx_cm.ctypes.data), ctypes.c_void_p(dist_cm.ctypes.data), n, k, 3, 5, 1.0, A, B, 1.0,
        30, 42, 0, 1, y_double.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    assert rc == 0, _lib.last_error()
    np.testing.assert_allclose(y_dev, y_float, atol=1e-5)
    np.testing.assert_allclose(y_double, y_float, atol=1e-5)


def test_one_based_indices(dev_golden):
    idx, dist = dev_golden["lowd_idx"], dev_golden["lowd_dist"]
    a = api.umap_graph_dump(idx, dist)
    b = api.umap_graph_dump(idx + 1, dist)
    np.testing.assert_array_equal(a["tails"], b["tails"])
    np.testing.assert_array_equal(a["weights"], b["weights"])


def test_fused_quality_vs_reference_cuda():
    """Default (in-place) mode end to end on a 50-D mixture: kNN preservation and
    label accuracy within 2% of the reference's own fused CUDA path, as means
    over six seeds (both runs are Hogwild; see quality.within_reference)."""
    from quality import knn_preservation, label_accuracy, within_reference

    if not O.ref_cuda_available():
        pytest.skip("oracle/_ref/libferef_cuda.so not built")
    spec = S.MixtureSpec(n=5000, dim=50, components=10, seed=11)
    x, labels = S.gaussian_mixture(spec)
    idx, dist = S.exact_knn(x, 15, device="cuda")
    q, qr, la, lar = [], [], [], []
    for seed in (42, 43, 44, 45, 46, 47):
        y = api.umap_knn(idx, dist, n_epochs=500, min_dist=0.1, seed=seed).Y
        yr = O.ref_cuda_umap_fused(idx, dist, n_epochs=500, spectral_n_iter=60, seed=seed)
        assert np.isfinite(y).all() and np.abs(y).max() <= 16.0
        q.append(knn_preservation(y, idx))
        qr.append(knn_preservation(yr, idx))
        la.append(label_accuracy(y, labels))
        lar.append(label_accuracy(yr, labels))
    ok_q, msg_q = within_reference(q, qr)
    ok_l, msg_l = within_reference(la, lar)
    print(f"fused UMAP: knn preservation {msg_q}; label acc {msg_l}")
    assert ok_l, msg_l
    assert ok_q, msg_q


def test_fused_invalid_arguments():
    n, k = 50, 5
    self_knn = np.repeat(np.arange(n, dtype=np.int32)[:, None], k, axis=1)
    with pytest.raises(api.CudaBackendError, match="invalid fused CUDA UMAP graph edge count"):
        api.umap_knn(self_knn, np.ones((n, k), np.float32), n_epochs=5)
    with pytest.raises(api.CudaBackendError, match="invalid CUDA UMAP graph edge count"):
        api.umap_graph_dump(self_knn, np.ones((n, k), np.float32))
