"""The C restatement (oracle/) against golden vectors from the reference's own CPU code.

These pin the checker itself: every GPU parity test compares the CUDA path with
this restatement, so it must reproduce the reference first.
"""
import numpy as np
import pytest

import oracle as O


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(np.asarray(b, np.float64)))


def test_tsne_affinities_bit_exact(tsne_golden):
    g = tsne_golden
    P = O.tsne_build_p(g["idx"], g["dist"], float(g["perplexity"]))
    assert np.array_equal(P.row_ptr, g["row_ptr"])
    assert np.array_equal(P.col, g["col"])
    assert np.array_equal(P.val, g["val"])
    assert abs(float(P.val.astype(np.float64).sum()) - 1.0) < 1e-4


def test_tsne_grid_policy(tsne_golden):
    assert O.tsne_grid_size(1000) == int(tsne_golden["grid"])
    assert [O.tsne_grid_size(n) for n in (9_999, 10_000, 49_999, 50_000, 1_000_000)] == [64, 128, 128, 256, 256]
    assert O.tsne_grid_size(10, 1000) == 512 and O.tsne_grid_size(10, 100) == 128


@pytest.mark.parametrize("state", [0, 1, 2])
def test_tsne_fft_gradient_matches_reference(tsne_golden, state):
    g = tsne_golden
    P = O.Csr(g["row_ptr"], g["col"], g["val"])
    y = g["states"][state]
    ex = float(g["exaggeration"][state])
    grad = O.tsne_gradient_fft(P, y, ex, int(g["grid"]))
    # Double-precision FFT vs the reference's float radix-2 FFT, whose twiddles
    # are formed by repeated multiplication: ~1e-4 relative at a wide layout.
    assert rel_l2(grad, g["grad_fft"][state]) < 5e-4


@pytest.mark.parametrize("state", [0, 1, 2])
def test_tsne_exact_gradient_bit_exact(tsne_golden, state):
    g = tsne_golden
    P = O.Csr(g["row_ptr"], g["col"], g["val"])
    grad = O.tsne_gradient_exact(P, g["states"][state], float(g["exaggeration"][state]))
    assert np.array_equal(grad, g["grad_exact"][state])


def test_tsne_update_bit_exact(tsne_golden):
    g = tsne_golden
    n = g["init"].shape[0]
    y, u, gn = O.tsne_update(g["states"][1], g["update_in"], g["gains_in"], g["grad_fft"][1],
                             n / 12.0, 0.8)
    assert np.array_equal(y, g["y_after_update"])
    assert np.array_equal(u, g["update_after"])
    assert np.array_equal(gn, g["gains_after"])


def test_tsne_kl_matches_reference(tsne_golden):
    g = tsne_golden
    P = O.Csr(g["row_ptr"], g["col"], g["val"])
    assert O.tsne_kl(P, g["y_run"]) == pytest.approx(float(g["kl_run"]), rel=1e-12)


def test_tsne_full_run_quality_matches_reference(tsne_golden):
    """End-to-end bar: the restated 750-iteration loop lands within 2% KL of the reference run."""
    g = tsne_golden
    P = O.Csr(g["row_ptr"], g["col"], g["val"])
    y = O.tsne_run(P, g["init"], grid_size=128)
    kl = O.tsne_kl(P, y)
    assert abs(kl - float(g["kl_run_g128"])) / float(g["kl_run_g128"]) < 0.02


def test_umap_graph_bit_exact(umap_golden):
    g = umap_golden
    gr = O.umap_graph(g["idx"], g["dist"])
    assert np.array_equal(gr.offsets, g["offsets"])
    assert np.array_equal(gr.neighbors, g["neighbors"])
    assert np.array_equal(gr.weights, g["weights"])
    assert np.array_equal(gr.epochs_per_sample, g["epochs_per_sample"])
    assert gr.max_weight == float(g["max_weight"])


@pytest.mark.parametrize("epochs,key", [(2, "replay2"), (10, "replay10")])
def test_umap_serial_replay_bit_exact(umap_golden, epochs, key):
    g = umap_golden
    heads = np.repeat(np.arange(g["offsets"].size - 1), np.diff(g["offsets"]))
    y = O.umap_replay_serial(heads, g["neighbors"], g["epochs_per_sample"], g["init"], 0, epochs,
                             epochs, seed=int(g["seed"]))
    assert np.array_equal(y, g[key])


def test_umap_delta_equals_serial_on_disjoint_edges():
    """With vertex-disjoint edges and no negatives, delta (Jacobi) and in-place orders agree."""
    rng = np.random.default_rng(0)
    n = 200
    perm = rng.permutation(n)
    heads, tails = perm[0::2].astype(np.int32), perm[1::2].astype(np.int32)
    eps = rng.uniform(1.0, 3.0, heads.size).astype(np.float32)
    y0 = rng.uniform(-10, 10, (n, 2)).astype(np.float32)
    for epoch in range(1, 6):
        d = O.umap_epoch_delta(heads, tails, eps, y0, epoch, 10, negative_sample_rate=0)
        s = O.umap_replay_serial(heads, tails, eps, y0, epoch, epoch + 1, 10, negative_sample_rate=0)
        assert np.array_equal(d, s)


def test_umap_scalar_helpers(umap_scalar_golden):
    g = umap_scalar_golden
    for bi, b in enumerate(g["bs"]):
        got = np.array([O.umap_powf(float(x), float(b)) for x in g["xs"]], np.float32)
        assert np.array_equal(got, g["pow_table"][bi])
    for pi, p in enumerate(g["periods"]):
        assert [O.umap_positive_samples(float(p), int(e)) for e in g["epochs"]] == g["pos"][pi].tolist()
        assert [O.umap_negative_samples(float(p), 5, int(e)) for e in g["epochs"]] == g["neg"][pi].tolist()
    got = [O.umap_negative_vertex(int(a[0]), int(a[1]), int(a[2]), int(a[3]), int(a[4]), int(a[5]))
           for a in g["hash_args"]]
    assert got == g["hashes"].tolist()
    for md, (a, b) in zip(g["ab_min_dist"], g["ab"]):
        assert O.umap_find_ab(1.0, float(md)) == (a, b)


# ------------------------------------------- device-KNN UMAP path (reference CUDA golden vectors)


def _row_lists(heads, tails, weights, n):
    order = np.lexsort((tails, heads))
    h, t, w = heads[order], tails[order], weights[order]
    bounds = np.searchsorted(h, np.arange(n + 1))
    return [(t[bounds[i]:bounds[i + 1]], w[bounds[i]:bounds[i + 1]]) for i in range(n)]


def test_umap_device_graph_against_reference_cuda(umap_device_golden, umap_golden):
    """The restated device graph against the reference's dump, row by row.  The
    low-dimensional graph has no full row, so every row must agree; in the hub
    graph full rows keep an arbitrary subset of incoming edges in the reference,
    so only their size and own KNN entries are compared.  Weights within 1e-4
    relative: the C library's expf differs from CUDA's in the last bits."""
    g = umap_device_golden
    for key, idx, dist in (("lowd", g["lowd_idx"], g["lowd_dist"]), ("hub", umap_golden["idx"], umap_golden["dist"])):
        n, k = idx.shape
        width = 2 * k
        nbr, w = O.umap_device_graph(idx, dist)
        coo = O.umap_pack_coo(nbr, w, rank_major=True)
        ours = _row_lists(coo["heads"], coo["tails"], coo["weights"], n)
        ref = _row_lists(g[f"{key}_heads"], g[f"{key}_tails"], g[f"{key}_weights"], n)
        full = 0
        for i, ((t, wt), (tr, wr)) in enumerate(zip(ours, ref)):
            if tr.size < width:
                np.testing.assert_array_equal(t, tr)
                np.testing.assert_allclose(wt, wr, rtol=1e-4)
            else:
                full += 1
                assert t.size == width
                own = np.unique(idx[i][idx[i] != i])
                assert np.isin(own, t).all() and np.isin(own, tr).all()
        assert (full == 0) == (key == "lowd")
        np.testing.assert_allclose(coo["epochs_per_sample"], 1.0 / np.maximum(coo["weights"], 1e-6), rtol=1e-6)


def test_umap_diffusion_start_against_reference_cuda(umap_device_golden):
    g = umap_device_golden
    for binary, key in ((False, "lowd_start"), (True, "lowd_start_binary")):
        nbr, w = O.umap_device_graph(g["lowd_idx"], g["lowd_dist"], binary=binary)
        y = O.umap_diffusion_init(nbr, w, int(g["seed"]), int(g["spectral_n_iter"]))
        np.testing.assert_allclose(y, g[key], atol=1e-6)


def test_umap_fused_jacobi_epochs_against_reference_cuda(umap_device_golden):
    """The reference's fused Jacobi run (3 epochs) replayed by the restatement on
    the reference's own edge list and start layout."""
    g = umap_device_golden
    y = g["lowd_start"].copy()
    for e in range(3):
        y = O.umap_epoch_delta(g["lowd_heads"], g["lowd_tails"], g["lowd_epochs_per_sample"], y, e, 3,
                               seed=int(g["seed"]), hash_key_is_tail=True)
    np.testing.assert_allclose(y, g["lowd_delta3"], atol=1e-3)


@pytest.mark.skipif(not O.ref_available(), reason="compiled reference not present")
def test_restatement_against_live_reference_fresh_seed():
    from fastembedr_b200 import synthetic as S

    x, _ = S.gaussian_mixture(S.MixtureSpec(n=600, dim=10, components=4, seed=99))
    idx, dist = S.exact_knn(x, 30)
    Pr = O.ref_tsne_build_p(idx, dist, 10.0)
    Po = O.tsne_build_p(idx, dist, 10.0)
    assert np.array_equal(Pr.val, Po.val) and np.array_equal(Pr.col, Po.col)
    y = np.random.default_rng(1).normal(0, 3, (600, 2)).astype(np.float32)
    assert rel_l2(O.tsne_gradient_fft(Po, y, 4.0, O.tsne_grid_size(600)),
                  O.ref_tsne_gradient_fft(Pr, y, 4.0)) < 5e-4
