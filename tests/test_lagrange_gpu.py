"""FIt-SNE box interpolation (Lagrange mode, fe_b200_tsne_set_interpolation /
FASTEMBEDR_B200_INTERPOLATION=lagrange) on the B200.

The reference has no such mode: its repulsion is bilinear on one G x G grid
(src/tsne_neighbors.cpp:1076-1182).  The mode is checked against
  * oracle.tsne_gradient_lagrange, a double-precision restatement of the
    published scheme (gradient within 1e-3 relative L2, Z within 1e-5);
  * the reference's own exact pairwise gradient (compute_gradient_pair_symmetric_f,
    src/tsne_neighbors.cpp:1014): at least as close to it as the reference's
    bilinear gradient at its own grid (both errors printed);
  * the exact-gradient t-SNE end to end (configuration 0, a committed
    fixture): final KL within 2% and kNN preservation within 5%.
"""
import os

import numpy as np
import pytest

import oracle as O
from fastembedr_b200 import api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu
THREADS = os.cpu_count() or 1


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(np.asarray(b, np.float64)))


@pytest.fixture(scope="module")
def cfg0():
    x, labels = S.gaussian_mixture(S.CONFIGS["tsne_10k"])
    idx, dist = S.exact_knn(x, 90, device="cuda")
    P = O.ref_tsne_build_p(idx, dist, 30.0, threads=THREADS) if O.ref_available() else O.tsne_build_p(idx, dist, 30.0)
    return idx, dist, labels, P


def _layouts(idx, dist, n):
    rng = np.random.default_rng(8)
    y_rand = rng.normal(0, 5, (n, 2)).astype(np.float32)
    with api.TsneSession.from_knn(idx, dist, perplexity=30.0, init=S.tsne_init(n)) as s:
        y_run = s.run(early_exaggeration_iter=250, n_iter=150)
    return [(y_rand, 12.0), (y_run, 1.0)]


def test_gradient_matches_restatement(cfg0):
    idx, dist, _, P = cfg0
    n = idx.shape[0]
    for y, ex in _layouts(idx, dist, n):
        for grid in (256, 512):
            with api.TsneSession.from_csr(P.row_ptr, P.col, P.val, y, grid_size=grid) as s:
                s.set_interpolation("lagrange")
                grad, z = s.gradient(ex)
            want, wz = O.tsne_gradient_lagrange(P, y, ex, grid, return_z=True)
            err = rel_l2(grad, want)
            print(f"Lagrange G={grid} (ex {ex}): rel-L2 vs restatement {err:.2e}, Z {z:.6g} vs {wz:.6g}")
            # Float FFT against the restatement's double one: at a converged
            # layout the gradient is a small residual of cancelling forces
            # (the bilinear path shows 5e-4 against its double restatement
            # there too); the bar is the gradient bar, 1e-3.
            assert err < 1e-3
            assert z == pytest.approx(wz, rel=1e-5)


def test_interpolation_error_against_the_exact_gradient(cfg0):
    idx, dist, _, P = cfg0
    n = idx.shape[0]
    G = O.tsne_grid_size(n)
    exact = O.ref_tsne_gradient_exact if O.ref_available() else O.tsne_gradient_exact
    for y, ex in _layouts(idx, dist, n):
        ge = exact(P, y, ex, threads=THREADS) if O.ref_available() else exact(P, y, ex)
        with api.TsneSession.from_csr(P.row_ptr, P.col, P.val, y, grid_size=2 * G) as s:
            s.set_interpolation("lagrange")
            gl, _ = s.gradient(ex)
        with api.TsneSession.from_csr(P.row_ptr, P.col, P.val, y, grid_size=G) as s:
            gb, _ = s.gradient(ex)
        el, eb = rel_l2(gl, ge), rel_l2(gb, ge)
        print(f"vs exact gradient (ex {ex}): Lagrange boxes (G={2 * G}) {el:.2e}, bilinear (G={G}) {eb:.2e}")
        # At a converged layout the gradient is a small residual of cancelling
        # forces, so both interpolations are far from it in relative terms
        # (measured: Lagrange 0.12, the reference's bilinear grid 0.87); the
        # bar is to be at least as accurate as the reference's scheme.
        assert el <= eb


def test_end_to_end_quality_vs_exact_tsne(cfg0, monkeypatch):
    """The interpolations approximate the exact t-SNE gradient, so the quality
    target of the Lagrange mode is the exact-gradient run (the restatement of
    the reference's exact pairwise gradient, same schedule and start:
    tests/golden/make_exact_tsne.py): final KL within 2% and 15-NN
    preservation within 5% of it.  The reference's bilinear run is printed
    beside it: at its coarse grid it lands 2% above the exact KL and inflates
    kNN preservation by 6% (4 seeds: Lagrange 2.744 / 0.161, reference
    bilinear 2.794 / 0.176, exact 2.733 / 0.166)."""
    import json

    from conftest import GOLDEN
    from quality import knn_preservation, tsne_kl

    idx, dist, _, P = cfg0
    n = idx.shape[0]
    init = S.tsne_init(n, seed=0)
    monkeypatch.setenv("FASTEMBEDR_B200_INTERPOLATION", "lagrange")
    y = api.opentsne_knn(idx, dist, perplexity=30.0, init=init).Y
    monkeypatch.delenv("FASTEMBEDR_B200_INTERPOLATION")
    exact = json.load(open(os.path.join(GOLDEN, "exact_tsne_cfg0.json")))
    kl, q = tsne_kl(P.row_ptr, P.col, P.val, y), knn_preservation(y, idx, 15)
    msg = f"N=10k Lagrange boxes: KL {kl:.4f}, kNN preservation {q:.4f}; exact t-SNE {exact['kl']:.4f} / " \
          f"{exact['knn_preservation_15']:.4f}"
    if O.ref_available():
        yr = O.ref_tsne_run(idx, dist, init=init, perplexity=30.0, threads=THREADS)
        msg += f"; reference bilinear {tsne_kl(P.row_ptr, P.col, P.val, yr):.4f} / {knn_preservation(yr, idx, 15):.4f}"
    print(msg)
    assert np.isfinite(y).all()
    assert abs(kl - exact["kl"]) / exact["kl"] < 0.02
    assert abs(q - exact["knn_preservation_15"]) / exact["knn_preservation_15"] < 0.05


def test_runs_are_bit_reproducible(cfg0):
    idx, dist, _, _ = cfg0
    n = idx.shape[0]
    outs = []
    for _ in range(2):
        with api.TsneSession.from_knn(idx, dist, perplexity=30.0, init=S.tsne_init(n), grid_size=256) as s:
            s.set_interpolation("lagrange")
            s.iterate(120, 12.0, 0.8, float(np.float32(n / 12.0)))
            outs.append(s.layout())
    assert np.array_equal(outs[0], outs[1])


def test_lagrange_needs_a_fine_enough_grid(cfg0):
    idx, dist, _, _ = cfg0
    with api.TsneSession.from_knn(idx, dist, perplexity=30.0, grid_size=128) as s:
        with pytest.raises(api.CudaBackendError, match="at least 256"):
            s.set_interpolation("lagrange")
