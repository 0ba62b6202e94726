"""openTSNE transform against a fixed reference layout on the B200
(fastembedr_cuda_landmark_tsne_from_device_knn) against the reference's own
CUDA implementation of the same entry point (src/embedding_cuda_kernels.cpp:3496-3610,
compiled unmodified in oracle/_ref), same device KNN and host inputs.

Every query is optimised on its own against the fixed reference, so the two
implementations follow the same per-query arithmetic; they differ in float
rounding only (the reference's build contracts multiply-adds, this library's
does not), and gains flip on the sign of near-zero gradients, which lets a
few trajectories part over hundreds of iterations.  Bars:
  * the affine start (no iterations) and one iteration: within 1e-4 of the
    layout's scale;
  * full transforms, exact repulsion and hashed negative samples: the median
    query within 1e-3 of the layout's scale, 99% within 1e-2, and the same
    kNN preservation (2%).
"""
import numpy as np
import pytest

import oracle as O
from fastembedr_b200 import api
from fastembedr_b200 import synthetic as S

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.ref_cuda_available(), reason="oracle/_ref/libferef_cuda.so not built")]


@pytest.fixture(scope="module")
def problem():
    import torch

    x, labels = S.gaussian_mixture(S.MixtureSpec(n=9000, dim=20, components=6, seed=11))
    ref, qry = x[:6000], x[6000:]
    # reference layout: a converged t-SNE of the reference points
    ridx, rdist = S.exact_knn(ref, 45)
    ref_layout = api.opentsne_knn(ridx, rdist, perplexity=15.0, n_iter=300, early_exaggeration_iter=100).Y
    # queries' KNN into the reference
    d2 = ((qry[:, None, :].astype(np.float64) - ref[None].astype(np.float64)) ** 2).sum(-1)
    qidx = np.argsort(d2, 1)[:, :30].astype(np.int32)
    qdist = np.sqrt(np.take_along_axis(d2, qidx, 1)).astype(np.float32)
    d_idx = torch.from_numpy(np.ascontiguousarray(qidx.T)).cuda()  # column-major n_query x k
    d_dist = torch.from_numpy(np.ascontiguousarray(qdist.T)).cuda()
    return {"ref": ref, "qry": qry, "layout": ref_layout, "qidx": qidx, "qdist": qdist, "d_idx": d_idx,
            "d_dist": d_dist, "labels": labels[6000:], "ref_labels": labels[:6000]}


def _both(pb, **kw):
    ours = api.landmark_tsne_transform(pb["qidx"], pb["qdist"], pb["ref"], pb["qry"], pb["layout"], **kw)
    kw.setdefault("n_negatives", pb["ref"].shape[0] if pb["ref"].shape[0] <= kw.get("exact_repulsion_threshold", 4096)
                  else 256)
    theirs = O.ref_cuda_landmark_tsne(pb["d_idx"].data_ptr(), pb["d_dist"].data_ptr(), 0, pb["ref"], pb["qry"],
                                      pb["layout"], pb["qidx"].shape[1], **kw)
    scale = float(np.abs(pb["layout"]).max())
    return ours, theirs, scale


def test_affine_start_matches_reference(problem):
    ours, theirs, scale = _both(problem, n_iter=0, early_exaggeration_iter=0)
    err = np.abs(ours - theirs).max() / scale
    print(f"affine start: max |diff| / scale {err:.2e}")
    assert np.isfinite(ours).all()
    assert err < 1e-4


@pytest.mark.parametrize("exact", [True, False])
def test_one_iteration_matches_reference(problem, exact):
    kw = dict(n_iter=1, early_exaggeration_iter=0)
    if not exact:
        kw.update(exact_repulsion_threshold=100, n_negatives=64)
    ours, theirs, scale = _both(problem, **kw)
    err = np.abs(ours - theirs).max() / scale
    print(f"one iteration ({'exact' if exact else 'sampled'}): max |diff| / scale {err:.2e}")
    assert err < 1e-4


@pytest.mark.parametrize("exact", [True, False])
def test_full_transform_matches_reference(problem, exact):
    from quality import knn_preservation

    kw = dict(n_iter=250, early_exaggeration_iter=50)
    if not exact:
        kw.update(exact_repulsion_threshold=100, n_negatives=64)
    ours, theirs, scale = _both(problem, **kw)
    d = np.linalg.norm(ours - theirs, axis=1) / scale
    print(f"full transform ({'exact' if exact else 'sampled'}): median {np.median(d):.2e}, "
          f"99th percentile {np.quantile(d, 0.99):.2e}, max {d.max():.2e}")
    assert np.isfinite(ours).all()
    assert np.median(d) < 1e-3
    assert np.quantile(d, 0.99) < 1e-2
    # Placement quality: each query's nearest reference points in the layout
    # against its KNN in the data.
    full_o = np.vstack([problem["layout"], ours])
    full_t = np.vstack([problem["layout"], theirs])
    n_ref = problem["ref"].shape[0]
    rows = np.arange(n_ref, full_o.shape[0])
    knn = np.full((full_o.shape[0], problem["qidx"].shape[1]), 0, np.int32)
    knn[n_ref:] = problem["qidx"]
    q_o = knn_preservation(full_o, knn, 15, rows=rows)
    q_t = knn_preservation(full_t, knn, 15, rows=rows)
    print(f"kNN preservation of the queries: {q_o:.4f} vs reference {q_t:.4f}")
    assert q_o >= 0.98 * q_t


def test_rejects_bad_arguments(problem):
    with pytest.raises(api.CudaBackendError, match="invalid CUDA landmark t-SNE"):
        api.landmark_tsne_transform(problem["qidx"], problem["qdist"], problem["ref"], problem["qry"],
                                    problem["layout"], perplexity=-1.0)
