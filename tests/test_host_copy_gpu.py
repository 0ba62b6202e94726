"""Host -> device copies of large pageable inputs (fe::h2d_copy).

Inputs of 16 MB or more go up in 4 MB chunks that several host threads copy
into pinned slots.  The runs are deterministic, so a call fed from pageable
host arrays must reproduce bit for bit the same call fed from device memory,
and the same call with staging switched off (FASTEMBEDR_B200_H2D_THREADS=1,
one direct cudaMemcpyAsync).  The sizes are chosen so that the last chunk is
partial.
"""
import numpy as np
import pytest

from fastembedr_b200 import api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def knn_61k():
    x, _ = S.gaussian_mixture(S.CONFIGS["tsne_70k"])
    x = x[:61_000]
    idx, dist = S.exact_knn(x, 90, device="cuda")
    assert idx.nbytes >= 16 << 20 and idx.nbytes % (4 << 20) != 0
    return idx, dist


def test_tsne_staged_host_inputs_match_device_and_direct(knn_61k, monkeypatch):
    import torch

    idx, dist = knn_61k
    n = idx.shape[0]
    init = S.tsne_init(n, seed=1)
    kw = dict(perplexity=30.0, init=init, early_exaggeration_iter=40, n_iter=40)
    staged = api.opentsne_knn(idx, dist, **kw).Y
    device = api.opentsne_knn(torch.from_numpy(idx).cuda(), torch.from_numpy(dist).cuda(), **kw).Y
    monkeypatch.setenv("FASTEMBEDR_B200_H2D_THREADS", "1")
    direct = api.opentsne_knn(idx, dist, **kw).Y
    assert np.isfinite(staged).all()
    assert np.array_equal(staged, device)
    assert np.array_equal(staged, direct)


def test_umap_graph_from_staged_host_knn_matches_direct(knn_61k, monkeypatch):
    """The graph build is deterministic (one radix sort and run-length union),
    so the dumped COO graph is bit-identical whichever way the KNN went up."""
    idx, dist = knn_61k
    staged = api.umap_graph_dump(idx, dist.astype(np.float64))
    monkeypatch.setenv("FASTEMBEDR_B200_H2D_THREADS", "1")
    direct = api.umap_graph_dump(idx, dist.astype(np.float64))
    assert staged.keys() == direct.keys()
    for key in staged:
        assert np.array_equal(np.asarray(staged[key]), np.asarray(direct[key])), key


def test_umap_coo_staged_edges_match_direct(monkeypatch):
    """Jacobi epochs add their deltas with float atomics, so two runs agree to
    rounding only; a misplaced chunk of heads, tails or periods would move
    points by whole units."""
    rng = np.random.default_rng(11)
    n, e = 200_000, 4_500_001  # 18 MB per edge array
    heads = rng.integers(0, n, e, dtype=np.int32)
    tails = rng.integers(0, n, e, dtype=np.int32)
    weights = rng.random(e, dtype=np.float32)
    eps = (1.0 / np.maximum(weights, 1e-3)).astype(np.float32)
    init = rng.uniform(-10, 10, (n, 2)).astype(np.float32)
    kw = dict(n_epochs=3, optimizer_mode=1)
    staged = api.umap_optimize_coo(heads, tails, weights, eps, init, **kw)
    monkeypatch.setenv("FASTEMBEDR_B200_H2D_THREADS", "1")
    direct = api.umap_optimize_coo(heads, tails, weights, eps, init, **kw)
    assert np.isfinite(staged).all()
    assert np.abs(staged - init).max() > 1e-2
    diff = float(np.abs(staged - direct).max())
    print(f"COO UMAP staged vs direct copies: max |diff| {diff:.2e}")
    assert diff < 1e-4
