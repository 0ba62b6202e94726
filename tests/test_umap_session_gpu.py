"""UMAP sessions (fe_b200_umap_*) on the B200, through the C ABI.

A session runs the device-KNN UMAP path of
fastembedr_cuda_umap_from_device_knn_spectral_float in pieces, so it must give
that entry point's graph, start and schedule:

  * its edge list is the graph-dump entry point's rank-major COO list;
  * its sample counts are the epoch kernel's schedules summed exactly
    (positives over epochs [b, e) telescope to floor((e-1)/p) - floor((b-1)/p));
  * a Jacobi run split into epoch ranges reaches the one-shot entry point's
    quality (both accumulate deltas with float atomics, so they agree
    statistically, not bit for bit).
"""
import numpy as np
import pytest

from fastembedr_b200 import api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mixture():
    spec = S.MixtureSpec(n=5000, dim=50, components=10, seed=11)
    x, labels = S.gaussian_mixture(spec)
    idx, dist = S.exact_knn(x, 15, device="cuda")
    return idx, dist, labels


def test_session_graph_is_the_graph_dump(mixture):
    idx, dist, _ = mixture
    dump = api.umap_graph_dump(idx, dist)
    with api.UmapSession.from_knn(idx, dist) as s:
        g = s.graph()
        assert s.info()["n_edges"] == dump["heads"].size
    assert np.array_equal(g["heads"], dump["heads"])
    assert np.array_equal(g["tails"], dump["tails"])
    np.testing.assert_allclose(g["epochs_per_sample"], dump["epochs_per_sample"], rtol=1e-5)


def _floors(p, epoch):
    if epoch <= 0:
        return np.zeros(p.size, np.int64)
    return np.floor(np.float32(epoch) / p).astype(np.int64)


def test_sample_counts_match_the_schedule(mixture):
    idx, dist, _ = mixture
    with api.UmapSession.from_knn(idx, dist) as s:
        p = s.graph()["epochs_per_sample"].astype(np.float32)
        for b, e in ((0, 200), (0, 1), (17, 91)):
            pos, neg = s.count_samples(b, e, 5)
            want = int((_floors(p, e - 1) - _floors(p, max(b, 1) - 1)).sum())
            assert pos == want, (b, e, pos, want)
            assert neg >= 0
        pos, neg = s.count_samples(0, 200, 0)
        assert neg == 0 and pos > 0


def test_split_jacobi_run_matches_one_shot_quality(mixture):
    """A run split into epoch ranges reaches the one-shot call's quality.  Jacobi
    epochs sum per-vertex moves with float atomics, so single runs at n = 5000
    differ by a few percent in kNN preservation; the bar is on means over
    seeds (3% plus two standard errors of the difference)."""
    from quality import knn_preservation, label_accuracy, within_reference

    idx, dist, labels = mixture
    q1, q2, l1, l2 = [], [], [], []
    for seed in (42, 43, 44, 45):
        one = api.umap_knn(idx, dist, n_epochs=200, min_dist=0.1, seed=seed, optimizer_mode=1).Y
        with api.UmapSession.from_knn(idx, dist, seed=seed) as s:
            for b, e in ((0, 60), (60, 61), (61, 200)):
                s.run(b, e, 200, min_dist=0.1, seed=seed, optimizer_mode=1)
            y = s.layout()
        assert np.isfinite(y).all() and np.abs(y).max() <= 16.0
        q1.append(knn_preservation(one, idx))
        q2.append(knn_preservation(y, idx))
        l1.append(label_accuracy(one, labels))
        l2.append(label_accuracy(y, labels))
    ok_q, msg_q = within_reference(q2, q1, rel=0.03)
    ok_l, msg_l = within_reference(l2, l1, rel=0.03)
    assert ok_q, msg_q
    assert ok_l, msg_l


def test_session_rejects_bad_ranges(mixture):
    idx, dist, _ = mixture
    with api.UmapSession.from_knn(idx, dist) as s:
        with pytest.raises(api.CudaBackendError, match="invalid UMAP epoch range"):
            s.run(5, 4, 200)
        with pytest.raises(api.CudaBackendError, match="invalid UMAP epoch range"):
            s.run(0, 201, 200)
