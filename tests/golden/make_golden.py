"""Generate the golden fixtures in this folder from the reference's own CPU code.

The reference ships no golden vectors for the optimizer path, so these are
produced by running the reference's CPU implementation (compiled unmodified
into ``oracle/_ref`` by ``oracle/Makefile``) on seeded synthetic inputs.  Run
from the repository root, where the reference sources are present:

    python tests/golden/make_golden.py

Outputs (compressed .npz, a few hundred KB each):
  tsne_small.npz  -- KNN input, symmetric P (build_tsne_probabilities_float),
                     FFT-grid and exact gradients at three layouts, one update
                     step, a 750-iteration run from a fixed init and its KL.
  umap_small.npz  -- KNN input, fuzzy-union CSR graph (umap_graph_csr_float_cpp),
                     sequential COO replays (fast_knn_umap_coo_replay_cpp,
                     n_threads = 1) after 2 and 10 epochs.
  umap_scalar.npz -- umap_powf_fast, the positive/negative schedules and the
                     negative-sample hash on tables of arguments.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402
from fastembedr_b200 import synthetic as S  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def ensemble_inits(init, members: int = 8, seed: int = 2024, scale: float = 1e-9):
    """Deterministic tiny perturbations of `init` (the tests rebuild the same set)."""
    rng = np.random.default_rng(seed)
    return [(init + rng.normal(0.0, scale, init.shape)).astype(np.float32) for _ in range(members)]


def tsne_small() -> None:
    n, k, perp = 1000, 45, 15.0
    x, _ = S.gaussian_mixture(S.MixtureSpec(n=n, dim=20, components=5, seed=11))
    idx, dist = S.exact_knn(x, k)
    P = O.ref_tsne_build_p(idx, dist, perp)
    grid = O.ref_tsne_grid_size(n)
    init = S.tsne_init(n, seed=5)
    # Layout states: the init, 50 early-exaggeration iterations, 400 iterations.
    y0 = O.tsne_zero_mean(init)
    y50 = O.ref_tsne_run(idx, dist, init=init, perplexity=perp, early_exaggeration_iter=50, n_iter=0)
    y400 = O.ref_tsne_run(idx, dist, init=init, perplexity=perp, early_exaggeration_iter=250,
                          n_iter=150)
    states = np.stack([y0, y50, y400])
    ex = np.array([12.0, 12.0, 1.0], np.float32)
    g_fft = np.stack([O.ref_tsne_gradient_fft(P, s, float(e)) for s, e in zip(states, ex)])
    g_exact = np.stack([O.ref_tsne_gradient_exact(P, s, float(e)) for s, e in zip(states, ex)])
    # One update from state 1 with non-trivial optimizer state.
    rng = np.random.default_rng(3)
    upd0 = rng.normal(0, 0.1, size=(n, 2)).astype(np.float32)
    gains0 = rng.uniform(0.01, 3.0, size=(n, 2)).astype(np.float32)
    y_u, upd_u, gains_u = O.ref_tsne_update(y50, upd0, gains0, g_fft[1], n / 12.0, 0.8)
    y_run = O.ref_tsne_run(idx, dist, init=init, perplexity=perp)
    kl_run = O.ref_tsne_kl(P, y_run)
    # At n = 1000 the default 64-node grid is too coarse for the late layout:
    # the interpolated normaliser Z decays towards zero and runs become
    # ill-conditioned.  End-to-end comparisons use a 128-node grid instead
    # (FASTEMBEDR_TSNE_FFT_GRID=128, honoured by the reference as well).
    y_run_g128 = O.ref_tsne_run(idx, dist, init=init, perplexity=perp, grid_override=128)
    kl_run_g128 = O.ref_tsne_kl(P, y_run_g128)
    # The dynamics are chaotic at this size: a 1e-9 change of the init moves
    # the final KL by a few percent.  The end-to-end bar is therefore applied
    # to the mean over an ensemble of perturbed inits (ensemble_inits()).
    kl_ensemble_g128 = np.array([
        O.ref_tsne_kl(P, O.ref_tsne_run(idx, dist, init=y0, perplexity=perp, grid_override=128))
        for y0 in ensemble_inits(init)])
    np.savez_compressed(
        os.path.join(OUT, "tsne_small.npz"),
        idx=idx, dist=dist, perplexity=np.float64(perp), grid=np.int32(grid),
        row_ptr=P.row_ptr, col=P.col, val=P.val, states=states, exaggeration=ex,
        grad_fft=g_fft, grad_exact=g_exact, update_in=upd0, gains_in=gains0,
        y_after_update=y_u, update_after=upd_u, gains_after=gains_u, init=init,
        y_run=y_run, kl_run=np.float64(kl_run), y_run_g128=y_run_g128,
        kl_run_g128=np.float64(kl_run_g128), kl_ensemble_g128=kl_ensemble_g128)


def umap_small() -> None:
    n, k = 1000, 15
    x, _ = S.gaussian_mixture(S.MixtureSpec(n=n, dim=20, components=5, seed=12))
    idx, dist = S.exact_knn(x, k)
    g = O.ref_umap_graph(idx, dist)
    heads = g.heads()
    init = S.umap_random_init(n, seed=7)
    rep2 = O.ref_umap_coo_replay(heads, g.neighbors, g.weights, g.epochs_per_sample, init, 2)
    rep10 = O.ref_umap_coo_replay(heads, g.neighbors, g.weights, g.epochs_per_sample, init, 10)
    np.savez_compressed(
        os.path.join(OUT, "umap_small.npz"),
        idx=idx, dist=dist, offsets=g.offsets, neighbors=g.neighbors, weights=g.weights,
        epochs_per_sample=g.epochs_per_sample, max_weight=np.float32(g.max_weight),
        init=init, replay2=rep2, replay10=rep10, seed=np.int32(42))


def umap_scalar() -> None:
    rng = np.random.default_rng(21)
    xs = np.concatenate([rng.uniform(1e-7, 1e-3, 300), rng.uniform(1e-3, 10, 400),
                         rng.uniform(10, 1e4, 300)]).astype(np.float32)
    bs = np.array([0.8950608781227859, 0.8006377738365004, 1.3341669931033755], np.float32)
    pow_table = np.array([[O.ref_umap_powf(float(x), float(b)) for x in xs] for b in bs], np.float32)
    periods = np.concatenate([[1.0], rng.uniform(1.0, 50.0, 200)]).astype(np.float32)
    epochs = np.arange(0, 60, dtype=np.int32)
    pos = np.array([[O.ref_umap_positive_samples(float(p), int(e)) for e in epochs] for p in periods],
                   np.int32)
    neg = np.array([[O.ref_umap_negative_samples(float(p), 5, int(e)) for e in epochs]
                    for p in periods], np.int32)
    args = np.stack([rng.integers(2, 5_000_000, 500), rng.integers(0, 2**31 - 1, 500),
                     rng.integers(0, 500, 500), rng.integers(0, 5_000_000, 500),
                     rng.integers(0, 60_000_000, 500), rng.integers(0, 30, 500)], 1).astype(np.int64)
    args[:, 2] = np.minimum(args[:, 2], 499)
    args[:, 3] = args[:, 3] % args[:, 0]
    hashes = np.array([O.ref_umap_negative_vertex(int(a[0]), int(a[1]), int(a[2]), int(a[3]),
                                                  int(a[4]), int(a[5])) for a in args], np.int32)
    ab = np.array([O.ref_find_ab(1.0, md) for md in (0.01, 0.1, 0.5, 0.25)], np.float64)
    np.savez_compressed(os.path.join(OUT, "umap_scalar.npz"), xs=xs, bs=bs, pow_table=pow_table,
                        periods=periods, epochs=epochs, pos=pos, neg=neg, hash_args=args,
                        hashes=hashes, ab_min_dist=np.array([0.01, 0.1, 0.5, 0.25]), ab=ab)


if __name__ == "__main__":
    if not O.ref_available():
        O.build()
    tsne_small()
    umap_small()
    umap_scalar()
    for f in sorted(os.listdir(OUT)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(OUT, f)))
