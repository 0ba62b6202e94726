"""Sharded UMAP sessions on B200s, one process per GPU, through the C ABI.

Each rank owns a block of vertices and the edges touching it, applies the
moves of its own vertices and all-gathers the blocks after every epoch.  In
the Jacobi mode that is the unsharded epoch, so each sharded Jacobi epoch, started from the layout the
unsharded session holds, must match that session's epoch to within the
float-atomic summation order (1e-4, the bar of the single-epoch parity tests;
chained epochs would amplify those last-bit differences); in the default
Hogwild mode a rank sees the other ranks' moves one epoch late, so the bar
there is end-to-end quality.

The two-rank tests need two GPUs and are skipped on a one-GPU box.
"""
import os
import subprocess
import sys

if __name__ == "__main__":  # a rank process of the two-GPU tests
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import numpy as np
import pytest

from fastembedr_b200 import api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu

N, K, N_EPOCHS, JACOBI_EPOCHS = 5000, 15, 200, 5
TOL = 1e-4


def _problem_arrays():
    x, labels = S.gaussian_mixture(S.MixtureSpec(n=N, dim=50, components=10, seed=11))
    idx, dist = S.exact_knn(x, K)
    return idx, dist, labels


def run_session(idx, dist, shard=None, mode=1, epochs=JACOBI_EPOCHS):
    """The session's diffusion start, then `epochs` epochs of a 200-epoch schedule."""
    with api.UmapSession.from_knn(idx, dist, seed=42) as s:
        if shard is not None:
            s.shard(*shard)
        s.run(0, epochs, N_EPOCHS, min_dist=0.1, seed=42, optimizer_mode=mode)
        return s.layout()


def jacobi_epoch_errors(idx, dist, shard):
    """Epochs 1 .. JACOBI_EPOCHS, each run by an unsharded and a sharded session
    from the unsharded session's layout: the largest difference per epoch."""
    errors = []
    with api.UmapSession.from_knn(idx, dist, seed=42) as plain, \
            api.UmapSession.from_knn(idx, dist, seed=42) as sharded:
        sharded.shard(*shard)
        for e in range(1, JACOBI_EPOCHS + 1):
            sharded.set_layout(plain.layout())
            plain.run(e, e + 1, N_EPOCHS, min_dist=0.1, seed=42, optimizer_mode=1)
            sharded.run(e, e + 1, N_EPOCHS, min_dist=0.1, seed=42, optimizer_mode=1)
            errors.append(float(np.abs(sharded.layout() - plain.layout()).max()))
    return np.asarray(errors)


@pytest.fixture(scope="module")
def problem(tmp_path_factory):
    idx, dist, labels = _problem_arrays()
    path = tmp_path_factory.mktemp("umap_shard") / "problem.npz"
    np.savez(path, idx=idx, dist=dist, labels=labels)
    return str(path)


def test_one_rank_shard_matches_unsharded_jacobi(problem):
    p = np.load(problem)
    errors = jacobi_epoch_errors(p["idx"], p["dist"], (api.nccl_unique_id(), 1, 0))
    assert errors.max() < TOL, errors


def test_shard_rejects_bad_ranks(problem):
    p = np.load(problem)
    with api.UmapSession.from_knn(p["idx"], p["dist"]) as s:
        with pytest.raises(api.CudaBackendError, match="nranks"):
            s.shard(api.nccl_unique_id(), 2, 5)


def _gpu_count():
    import torch

    return torch.cuda.device_count()


def _run_ranks(problem, tmp_path, mode, epochs):
    uid = api.nccl_unique_id()
    procs = []
    for rank in range(2):
        out = tmp_path / f"umap_rank{rank}_{mode}.npy"
        env = dict(os.environ, NCCL_NVLS_ENABLE="0")
        cmd = [sys.executable, __file__, problem, uid.hex(), "2", str(rank), str(out), str(mode), str(epochs)]
        procs.append((out, subprocess.Popen(cmd, env=env)))
    try:
        codes = [p.wait(timeout=300) for _, p in procs]
    finally:
        for _, p in procs:  # a rank left waiting for a failed peer is ended here
            if p.poll() is None:
                p.kill()
                p.wait()
    assert codes == [0, 0], codes
    return [np.load(out) for out, _ in procs]


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_two_ranks_jacobi_match_unsharded(problem, tmp_path):
    for errors in _run_ranks(problem, tmp_path, 1, JACOBI_EPOCHS):
        assert errors.max() < TOL, errors


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_two_ranks_hogwild_quality(problem, tmp_path):
    from quality import knn_preservation, label_accuracy

    p = np.load(problem)
    plain = run_session(p["idx"], p["dist"], mode=0, epochs=N_EPOCHS)
    ranks = _run_ranks(problem, tmp_path, 0, N_EPOCHS)
    assert np.array_equal(ranks[0], ranks[1])  # every rank ends with the gathered layout
    y = ranks[0]
    assert np.isfinite(y).all() and np.abs(y).max() <= 16.0
    assert knn_preservation(y, p["idx"]) >= 0.97 * knn_preservation(plain, p["idx"])
    assert label_accuracy(y, p["labels"]) >= 0.97 * label_accuracy(plain, p["labels"])


def _rank_main(problem, uid_hex, nranks, rank, out, mode, epochs):
    import torch

    torch.cuda.set_device(rank)
    p = np.load(problem)
    shard = (bytes.fromhex(uid_hex), nranks, rank)
    if mode == 1:  # per-epoch errors against an unsharded session on this rank's GPU
        np.save(out, jacobi_epoch_errors(p["idx"], p["dist"], shard))
    else:
        np.save(out, run_session(p["idx"], p["dist"], shard=shard, mode=mode, epochs=epochs))


if __name__ == "__main__":
    _rank_main(sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4]), sys.argv[5], int(sys.argv[6]),
               int(sys.argv[7]))
