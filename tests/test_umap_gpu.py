"""UMAP parity on the B200: the CUDA COO optimizer (through the C ABI) against the oracle.

Bars: one epoch replayed with the same edge schedule and negative-sample
indices matches the oracle within 1e-4 absolute (Jacobi/delta mode, the
deterministic form); the in-place mode equals the sequential reference replay
where edges do not interact; end-to-end quality (kNN preservation) within 2%
of the reference CPU optimizer.
"""
import numpy as np
import pytest

import oracle as O
from fastembedr_b200 import api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu

A, B = 1.5769434601962196, 0.8950608781227859


@pytest.fixture(scope="module")
def cfg1():
    """Configuration 1 (N = 70k, k = 15 fuzzy union, random init U(-10, 10))."""
    x, labels = S.gaussian_mixture(S.CONFIGS["umap_70k"])
    idx, dist = S.exact_knn(x, 15, device="cuda")
    g = O.umap_graph(idx, dist)
    return idx, dist, g, labels


def _coo(g):
    return g.heads(), g.neighbors, g.weights, g.epochs_per_sample


@pytest.mark.parametrize("epoch", [1, 2, 7, 100])
@pytest.mark.parametrize("key_tail", [False, True])
def test_one_epoch_delta_matches_oracle_golden(umap_golden, epoch, key_tail):
    g = umap_golden
    heads = np.repeat(np.arange(g["offsets"].size - 1), np.diff(g["offsets"])).astype(np.int32)
    y0 = g["init"]
    got, _ = api.umap_epochs(heads, g["neighbors"], g["epochs_per_sample"], y0, epoch, epoch + 1, 200,
                             a=A, b=B, optimizer_mode=1, hash_key_is_tail=key_tail)
    want = O.umap_epoch_delta(heads, g["neighbors"], g["epochs_per_sample"], y0, epoch, 200, a=A, b=B,
                              hash_key_is_tail=key_tail)
    assert np.abs(got - want).max() < 1e-4


@pytest.mark.parametrize("epoch", [1, 3, 250])
def test_one_epoch_delta_matches_oracle_cfg1(cfg1, epoch):
    idx, dist, g, _ = cfg1
    heads, tails, _, eps = _coo(g)
    y0 = S.umap_random_init(idx.shape[0], seed=1)
    got, pos = api.umap_epochs(heads, tails, eps, y0, epoch, epoch + 1, 500, a=A, b=B, optimizer_mode=1)
    want = O.umap_epoch_delta(heads, tails, eps, y0, epoch, 500, a=A, b=B)
    assert np.abs(got - want).max() < 1e-4
    expected_pos = sum(O.umap_positive_samples(float(p), epoch) for p in eps[:2000])
    assert pos >= expected_pos


def test_positive_sample_count_matches_schedule(umap_golden):
    g = umap_golden
    heads = np.repeat(np.arange(g["offsets"].size - 1), np.diff(g["offsets"])).astype(np.int32)
    eps = g["epochs_per_sample"]
    _, pos = api.umap_epochs(heads, g["neighbors"], eps, g["init"], 0, 30, 30, optimizer_mode=1)
    want = sum(O.umap_positive_samples(float(p), e) for p in eps for e in range(30))
    assert pos == want


def test_inplace_equals_sequential_replay_on_disjoint_edges():
    rng = np.random.default_rng(0)
    n = 4000
    perm = rng.permutation(n)
    heads, tails = perm[0::2].astype(np.int32), perm[1::2].astype(np.int32)
    eps = rng.uniform(1.0, 3.0, heads.size).astype(np.float32)
    y0 = rng.uniform(-10, 10, (n, 2)).astype(np.float32)
    got, _ = api.umap_epochs(heads, tails, eps, y0, 0, 20, 20, negative_sample_rate=0, optimizer_mode=0)
    want = O.umap_replay_serial(heads, tails, eps, y0, 0, 20, 20, negative_sample_rate=0)
    assert np.abs(got - want).max() < 1e-5


def test_inplace_tracks_sequential_replay_golden(umap_golden):
    """Hogwild differs from the sequential reference replay only in update
    interleaving: per-point displacements after 10 epochs stay aligned."""
    g = umap_golden
    heads = np.repeat(np.arange(g["offsets"].size - 1), np.diff(g["offsets"])).astype(np.int32)
    got, _ = api.umap_epochs(heads, g["neighbors"], g["epochs_per_sample"], g["init"], 0, 10, 10,
                             a=A, b=B, optimizer_mode=0)
    assert np.isfinite(got).all()
    d_got = (got - g["init"]).ravel()
    d_ref = (g["replay10"] - g["init"]).ravel()
    corr = float(np.corrcoef(d_got, d_ref)[0, 1])
    assert corr > 0.8, corr


@pytest.mark.parametrize("mode", [0, 1])
def test_end_to_end_quality_vs_reference_cpu(cfg1, mode):
    """Default (in-place) mode: kNN preservation and label accuracy within 2% of
    the reference's CPU replay of the same COO schedule
    (fast_knn_umap_coo_replay_cpp, all host threads), as means over four random
    starts (both runs are Hogwild; see quality.within_reference).  The Jacobi
    mode is a different update order (all forces from the epoch-start layout);
    it is held to the label-accuracy bar and a looser preservation floor."""
    from quality import knn_preservation, label_accuracy, within_reference

    idx, dist, g, labels = cfg1
    heads, tails, w, eps = _coo(g)
    n = idx.shape[0]
    q, qr, la, lar = [], [], [], []
    for seed in (3, 4, 5, 6):
        init = S.umap_random_init(n, seed=seed)
        y = api.umap_optimize_coo(heads, tails, w, eps, init, n_epochs=500, min_dist=0.1, optimizer_mode=mode)
        assert np.isfinite(y).all() and np.abs(y).max() <= 16.0
        if O.ref_available():
            yr = O.ref_umap_coo_replay(heads, tails, w, eps, init, 500, min_dist=0.1, threads=8)
        else:
            yr = O.umap_replay_serial(heads, tails, eps, init, 0, 500, 500, a=A, b=B)
        q.append(knn_preservation(y, idx))
        qr.append(knn_preservation(yr, idx))
        la.append(label_accuracy(y, labels))
        lar.append(label_accuracy(yr, labels))
    ok_q, msg_q = within_reference(q, qr, rel=0.02 if mode == 0 else 0.25)
    ok_l, msg_l = within_reference(la, lar)
    print(f"mode {mode}: knn preservation {msg_q}; label acc {msg_l}")
    assert ok_l, msg_l
    assert ok_q, msg_q


def test_reference_default_key_is_edge_id(umap_golden, monkeypatch):
    """optimize_coo keys negatives on the edge id unless told otherwise."""
    g = umap_golden
    heads = np.repeat(np.arange(g["offsets"].size - 1), np.diff(g["offsets"])).astype(np.int32)
    out = api.umap_optimize_coo(heads, g["neighbors"], g["weights"], g["epochs_per_sample"], g["init"],
                                n_epochs=2, optimizer_mode=1)
    want = O.umap_epoch_delta(heads, g["neighbors"], g["epochs_per_sample"], g["init"], 1, 2, a=A, b=B)
    assert np.abs(out - want).max() < 1e-4


def test_umap_invalid_arguments():
    with pytest.raises(api.CudaBackendError, match="invalid CUDA COO UMAP"):
        api.umap_optimize_coo([0], [1], [1.0], [1.0], np.zeros((2, 2), np.float32), n_epochs=0)
