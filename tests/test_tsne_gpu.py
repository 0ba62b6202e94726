"""t-SNE parity on the B200: the CUDA path (through the C ABI) against the oracle.

Bars (from the parity definition of the optimizer path):
  * per-iteration gradient at an identical layout and P: relative L2 <= 1e-3;
  * affinities P: same sparsity pattern, values within float rounding of the
    expf/logf ulps (relative <= 1e-4);
  * end to end: final KL within 2% of the reference CPU run.
"""
import numpy as np
import pytest

import oracle as O
from fastembedr_b200 import api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def cfg0():
    """Configuration 0 (N = 10k, 10 equal components, k = 90, perplexity 30)."""
    x, labels = S.gaussian_mixture(S.CONFIGS["tsne_10k"])
    idx, dist = S.exact_knn(x, 90, device="cuda")
    return idx, dist, labels


def test_library_reports_b200():
    assert api.cuda_available()
    assert "sm_100a" in api.version()


def test_affinities_match_oracle(tsne_golden):
    g = tsne_golden
    with api.TsneSession.from_knn(g["idx"], g["dist"], perplexity=float(g["perplexity"]),
                                  init=g["init"]) as s:
        rp, col, val = s.p()
    assert np.array_equal(rp, g["row_ptr"])
    assert np.array_equal(col, g["col"])
    np.testing.assert_allclose(val, g["val"], rtol=1e-4, atol=0)


def test_affinities_match_oracle_cfg0(cfg0):
    idx, dist, _ = cfg0
    ref = O.tsne_build_p(idx, dist, 30.0)
    with api.TsneSession.from_knn(idx, dist, perplexity=30.0, init=S.tsne_init(idx.shape[0])) as s:
        rp, col, val = s.p()
    assert np.array_equal(rp, ref.row_ptr)
    assert np.array_equal(col, ref.col)
    assert rel_l2(val, ref.val) < 1e-5
    assert abs(val.astype(np.float64).sum() - 1.0) < 1e-4


@pytest.mark.parametrize("state", [0, 1, 2])
def test_gradient_matches_reference_golden(tsne_golden, state):
    """Gradient at the reference's own layouts vs the reference's own gradient."""
    g = tsne_golden
    y = g["states"][state]
    ex = float(g["exaggeration"][state])
    with api.TsneSession.from_csr(g["row_ptr"], g["col"], g["val"], y, grid_size=int(g["grid"])) as s:
        grad, z = s.gradient(ex)
    assert rel_l2(grad, g["grad_fft"][state]) < GRAD_TOL
    P = O.Csr(g["row_ptr"], g["col"], g["val"])
    ograd, oz = O.tsne_gradient_fft(P, y, ex, int(g["grid"]), return_z=True)
    assert rel_l2(grad, ograd) < 1e-4
    assert z == pytest.approx(oz, rel=1e-5)


@pytest.mark.parametrize("grid", [64, 128, 256, 512, 1024])
def test_gradient_grid_sizes(tsne_golden, grid):
    g = tsne_golden
    y = g["states"][2]
    P = O.Csr(g["row_ptr"], g["col"], g["val"])
    with api.TsneSession.from_csr(g["row_ptr"], g["col"], g["val"], y, grid_size=grid) as s:
        grad, _ = s.gradient(1.0)
    assert rel_l2(grad, O.tsne_gradient_fft(P, y, 1.0, grid)) < GRAD_TOL


def test_gradient_cfg0_layouts(cfg0):
    """N = 10k at the CPU grid (128): a random layout and a converged one."""
    idx, dist, _ = cfg0
    n = idx.shape[0]
    P = O.tsne_build_p(idx, dist, 30.0)
    G = O.tsne_grid_size(n)
    rng = np.random.default_rng(4)
    y_rand = rng.normal(0, 10, (n, 2)).astype(np.float32)
    with api.TsneSession.from_knn(idx, dist, perplexity=30.0, init=S.tsne_init(n)) as s:
        y_run = s.run(early_exaggeration_iter=250, n_iter=150)
    for y, ex in ((y_rand, 12.0), (y_run, 1.0), (y_run, 12.0)):
        with api.TsneSession.from_csr(P.row_ptr, P.col, P.val, y, grid_size=G) as s:
            grad, _ = s.gradient(ex)
        assert rel_l2(grad, O.tsne_gradient_fft(P, y, ex, G)) < GRAD_TOL


def test_one_iteration_matches_oracle_update(tsne_golden):
    """gradient + gains/momentum/clip update + re-centring for one iteration."""
    g = tsne_golden
    y = g["states"][1]
    n = y.shape[0]
    P = O.Csr(g["row_ptr"], g["col"], g["val"])
    G = int(g["grid"])
    lr = float(np.float32(n / 12.0))
    with api.TsneSession.from_csr(g["row_ptr"], g["col"], g["val"], y, grid_size=G) as s:
        s.set_state(g["update_in"], g["gains_in"])
        s.iterate(1, 12.0, 0.8, lr, 0.01, 5.0)
        y1 = s.layout()
        u1, g1 = s.state()
    grad = O.tsne_gradient_fft(P, O.tsne_zero_mean(y), 12.0, G)
    ey, eu, eg = O.tsne_update(O.tsne_zero_mean(y), g["update_in"], g["gains_in"], grad, lr, 0.8)
    assert rel_l2(u1, eu) < GRAD_TOL
    assert np.abs(y1 - ey).max() < 1e-3 * np.abs(eu).max() + 1e-6
    # Gains take discrete steps; allow a handful of sign flips at near-zero gradients.
    assert np.mean(np.abs(g1 - eg) > 1e-5) < 1e-3


def test_end_to_end_kl_within_2pct_of_reference(tsne_golden):
    g = tsne_golden
    P = O.Csr(g["row_ptr"], g["col"], g["val"])
    res = api.opentsne_knn(g["idx"], g["dist"], perplexity=float(g["perplexity"]), init=g["init"])
    assert res.config["optimizer"] == "opentsne_fitsne_fft_grid_native_cuda"
    assert res.config["repulsion"] == "fft_grid_cuda_cufft"
    kl = O.tsne_kl(P, res.Y)
    assert np.isfinite(res.Y).all()
    assert abs(kl - float(g["kl_run"])) / float(g["kl_run"]) < 0.02


def test_double_distances_and_one_based_indices(tsne_golden):
    g = tsne_golden
    import ctypes

    from fastembedr_b200 import _lib

    n, k = g["idx"].shape
    idx_cm = np.ascontiguousarray((g["idx"] + 1).T.astype(np.int32))
    dist_cm = np.ascontiguousarray(g["dist"].T.astype(np.float64))
    init = np.ascontiguousarray(g["init"], np.float32)
    out = np.zeros((n, 2), np.float32)
    L = _lib.load()
    rc = L.fastembedr_cuda_opentsne_fft_from_knn(
        ctypes.c_void_p(idx_cm.ctypes.data), ctypes.c_void_p(dist_cm.ctypes.data),
        init.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), 1, n, k, 2, float(g["perplexity"]),
        250, 500, 12.0, 1.0, 0.0, 1, 0.8, 0.8, 0.01, 5.0, 42, 1,
        out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    assert rc == 0, _lib.last_error()
    P = O.Csr(g["row_ptr"], g["col"], g["val"])
    assert abs(O.tsne_kl(P, out) - float(g["kl_run"])) / float(g["kl_run"]) < 0.02


def test_device_knn_entry_point(tsne_golden):
    import torch

    g = tsne_golden
    idx = torch.from_numpy(g["idx"]).cuda()
    dist = torch.from_numpy(g["dist"]).cuda()
    res = api.opentsne_knn(idx, dist, perplexity=float(g["perplexity"]), init=g["init"])
    P = O.Csr(g["row_ptr"], g["col"], g["val"])
    assert abs(O.tsne_kl(P, res.Y) - float(g["kl_run"])) / float(g["kl_run"]) < 0.02


def test_checkpoint_resume_is_exact(tsne_golden):
    g = tsne_golden
    n = g["init"].shape[0]
    lr = float(np.float32(n / 12.0))
    with api.TsneSession.from_csr(g["row_ptr"], g["col"], g["val"], g["init"]) as a:
        a.iterate(40, 12.0, 0.8, lr)
        y_full = None
        a.iterate(10, 12.0, 0.8, lr)
        y_full = a.layout()
    with api.TsneSession.from_csr(g["row_ptr"], g["col"], g["val"], g["init"]) as b:
        b.iterate(40, 12.0, 0.8, lr)
        y_mid, (u, gn) = b.layout(), b.state()
    with api.TsneSession.from_csr(g["row_ptr"], g["col"], g["val"], y_mid) as c:
        c.set_state(u, gn)
        c.iterate(10, 12.0, 0.8, lr)
        y_res = c.layout()
    # Resuming re-centres an already centred layout: identical up to float rounding.
    assert np.abs(y_res - y_full).max() < 1e-4 * max(1.0, np.abs(y_full).max())


def test_invalid_arguments_return_status_1():
    import ctypes

    from fastembedr_b200 import _lib

    L = _lib.load()
    out = np.zeros((10, 2), np.float32)
    idx = np.zeros(10 * 3, np.int32)
    dist = np.ones(10 * 3, np.float32)
    args = [ctypes.c_void_p(idx.ctypes.data), ctypes.c_void_p(dist.ctypes.data), None, 0, 10, 3, 3, 1.0,
            10, 10, 12.0, 1.0, 0.0, 1, 0.8, 0.8, 0.01, 5.0, 1, 0,
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))]
    assert L.fastembedr_cuda_opentsne_fft_from_knn_float(*args) == 1  # n_components = 3
    assert "invalid CUDA openTSNE" in _lib.last_error()
    args[6] = 2
    args[4] = 1
    assert L.fastembedr_cuda_opentsne_fft_from_knn_float(*args) == 1  # n = 1
    args[4] = 10
    args[0] = None
    assert L.fastembedr_cuda_opentsne_fft_from_knn_float(*args) == 1
    assert "null" in _lib.last_error()


def test_all_self_knn_reports_no_edges():
    n, k = 50, 3
    idx = np.tile(np.arange(n, dtype=np.int32)[:, None], (1, k))
    dist = np.zeros((n, k), np.float32)
    with pytest.raises(api.CudaBackendError, match="no non-self"):
        api.opentsne_knn(idx, dist, perplexity=1.0, init=np.zeros((n, 2), np.float32))
