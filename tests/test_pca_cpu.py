"""The PCA start restatement (oracle.pca_start) against scikit-learn's PCA.

The reference computes the PCA start of its PCA-initialised entry points with
RAFT's TSVD (src/embedding_cuda_kernels.cpp:3357-3495), which is not built in
the reference library here, so the restatement is pinned against an
independent implementation: scikit-learn's full-SVD PCA, whose sign rule
(svd_flip on U) also makes each component's largest-magnitude score positive.
"""
import numpy as np

import oracle as O
from fastembedr_b200 import synthetic as S


def _sklearn_start(x):
    from sklearn.decomposition import PCA

    s = PCA(n_components=2, svd_solver="full").fit_transform(x.astype(np.float64))
    n = s.shape[0]
    sd = s.std(0, ddof=1)
    return ((s - s.mean(0)) * (1e-4 / sd.max())).astype(np.float32)


def test_pca_start_matches_sklearn():
    x, _ = S.gaussian_mixture(S.MixtureSpec(n=3000, dim=20, components=5, seed=7))
    ours = O.pca_start(x)
    ref = _sklearn_start(x)
    assert ours.shape == (3000, 2)
    np.testing.assert_allclose(ours, ref, rtol=0, atol=1e-4 * 1e-4)  # 1e-4 of the layout's sd
    assert abs(float(ours.std(0, ddof=1).max()) - 1e-4) < 1e-9


def test_pca_start_sign_rule():
    x, _ = S.gaussian_mixture(S.MixtureSpec(n=500, dim=8, components=3, seed=1))
    for flip in (1.0, -1.0):
        y = O.pca_start(flip * x)
        for c in range(2):
            assert y[np.argmax(np.abs(y[:, c] - 0)), c] != 0
        # the start does not depend on the data's global sign
        np.testing.assert_allclose(y, O.pca_start(x), atol=1e-10)
