"""Exact-gradient t-SNE at configuration 0 (N = 10k) on the CPU: the quality
target of the Lagrange-box mode.

Runs the standard schedule (250 iterations at exaggeration 12, then 500 at 1,
momentum 0.8, learning rate n / exaggeration, the reference's gains / clip
update) with the exact pairwise gradient of the C restatement
(oracle.tsne_gradient_exact, the reference's compute_gradient_pair_symmetric_f,
src/tsne_neighbors.cpp:1014) from the standard start (seed 0), and records its
final exact KL and 15-NN preservation.  About 3 minutes on 8 cores.

    python tests/golden/make_exact_tsne.py   # -> tests/golden/exact_tsne_cfg0.json
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle as O  # noqa: E402
from fastembedr_b200 import synthetic as S  # noqa: E402


def main():
    x, _ = S.gaussian_mixture(S.CONFIGS["tsne_10k"])
    idx, dist = S.exact_knn_numpy(x, 90)
    P = O.tsne_build_p(idx, dist, 30.0)
    n = idx.shape[0]
    y = O.tsne_zero_mean(S.tsne_init(n, seed=0))
    upd, gains = np.zeros_like(y), np.ones_like(y)
    for it in range(750):
        ex = 12.0 if it < 250 else 1.0
        g = O.tsne_gradient_exact(P, y, ex)
        y, upd, gains = O.tsne_update(y, upd, gains, g, np.float32(n / ex), 0.8)
        y = O.tsne_zero_mean(y)
    d2 = ((y[:, None, :].astype(np.float64) - y[None]) ** 2).sum(-1)
    np.fill_diagonal(d2, np.inf)
    nn = np.argsort(d2, 1)[:, :15]
    knn15 = float((nn[:, :, None] == idx[:, None, :15]).any(-1).sum(1).mean() / 15)
    out = {"config": "tsne_10k", "seed": 0, "iterations": [250, 500], "kl": float(O.tsne_kl(P, y)),
           "knn_preservation_15": knn15}
    with open(os.path.join(HERE, "exact_tsne_cfg0.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(out)


if __name__ == "__main__":
    main()
