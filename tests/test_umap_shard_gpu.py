"""Sharded UMAP sessions on B200s, one process per GPU, through the C ABI.

Each rank owns a block of vertices and the edges touching it, applies the
moves of its own vertices and all-gathers the blocks (once per Jacobi epoch,
four times per Hogwild epoch).  In the Jacobi mode that is the unsharded epoch
exactly, so every sharded Jacobi epoch, started from a layout all ranks share,
must match the oracle's Jacobi epoch (a restatement of
embed_epoch_coo_delta_kernel + apply_delta_sanitize_layout_kernel,
src/embedding_cuda_kernels.cpp:3136-3222) within 1e-4, the bar of the
single-epoch parity tests.  In the default Hogwild mode a rank sees the other
ranks' moves up to a quarter of an epoch late, so the bar there is end-to-end
quality: kNN preservation and label accuracy within 2% (plus two standard
errors of the seed means) of unsharded runs, as for the fused path.

The two-rank tests need two GPUs and are skipped on a one-GPU box.
"""
import os
import subprocess
import sys

if __name__ == "__main__":  # a rank process of the two-GPU tests
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import numpy as np
import pytest

import oracle as O
from fastembedr_b200 import api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu

N, K, N_EPOCHS, JACOBI_EPOCHS = 5000, 15, 200, 5
TOL = 1e-4
SEEDS = (42, 43, 44)


def _problem_arrays():
    x, labels = S.gaussian_mixture(S.MixtureSpec(n=N, dim=50, components=10, seed=11))
    idx, dist = S.exact_knn(x, K)
    return idx, dist, labels


def run_session(idx, dist, shard=None, mode=1, epochs=JACOBI_EPOCHS, seed=42):
    """The session's diffusion start, then `epochs` epochs of a 200-epoch schedule."""
    with api.UmapSession.from_knn(idx, dist, seed=seed) as s:
        if shard is not None:
            s.shard(*shard)
        s.run(0, epochs, N_EPOCHS, min_dist=0.1, seed=seed, optimizer_mode=mode)
        return s.layout()


def jacobi_epoch_errors(idx, dist, shard):
    """Epochs 1 .. JACOBI_EPOCHS of a sharded session, each started from the
    oracle's layout of the previous epoch (the same on every rank): the
    largest difference to the oracle's epoch, per epoch."""
    a, b = api.find_ab_params(1.0, 0.1)
    errors = []
    with api.UmapSession.from_knn(idx, dist, seed=42) as s:
        g = s.graph()
        s.shard(*shard)
        y = S.umap_random_init(N, seed=5)
        for e in range(1, JACOBI_EPOCHS + 1):
            want = O.umap_epoch_delta(g["heads"], g["tails"], g["epochs_per_sample"], y, e, N_EPOCHS, a=a, b=b,
                                      seed=42, hash_key_is_tail=True)
            s.set_layout(y)
            s.run(e, e + 1, N_EPOCHS, min_dist=0.1, seed=42, optimizer_mode=1)
            errors.append(float(np.abs(s.layout() - want).max()))
            y = want
    return np.asarray(errors)


@pytest.fixture(scope="module")
def problem(tmp_path_factory):
    idx, dist, labels = _problem_arrays()
    path = tmp_path_factory.mktemp("umap_shard") / "problem.npz"
    np.savez(path, idx=idx, dist=dist, labels=labels)
    return str(path)


def test_one_rank_shard_matches_oracle_jacobi(problem):
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
    # One communicator per sharded session the ranks create (one per seed in
    # the Hogwild test); an id serves one communicator.
    uids = ",".join(api.nccl_unique_id().hex() for _ in SEEDS)
    procs = []
    for rank in range(2):
        out = tmp_path / f"umap_rank{rank}_{mode}.npy"
        env = dict(os.environ, NCCL_NVLS_ENABLE="0")
        cmd = [sys.executable, __file__, problem, uids, "2", str(rank), str(out), str(mode), str(epochs)]
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
def test_two_ranks_jacobi_match_oracle(problem, tmp_path):
    for errors in _run_ranks(problem, tmp_path, 1, JACOBI_EPOCHS):
        assert errors.max() < TOL, errors


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_two_ranks_hogwild_quality(problem, tmp_path):
    from quality import knn_preservation, label_accuracy, within_reference

    p = np.load(problem)
    ranks = _run_ranks(problem, tmp_path, 0, N_EPOCHS)
    assert np.array_equal(ranks[0], ranks[1])  # every rank ends with the gathered layouts
    q, qr, la, lar = [], [], [], []
    for i, seed in enumerate(SEEDS):
        y = ranks[0][i]
        assert np.isfinite(y).all() and np.abs(y).max() <= 16.0
        plain = run_session(p["idx"], p["dist"], mode=0, epochs=N_EPOCHS, seed=seed)
        q.append(knn_preservation(y, p["idx"]))
        qr.append(knn_preservation(plain, p["idx"]))
        la.append(label_accuracy(y, p["labels"]))
        lar.append(label_accuracy(plain, p["labels"]))
    ok_q, msg_q = within_reference(q, qr)
    ok_l, msg_l = within_reference(la, lar)
    print(f"sharded UMAP: knn preservation {msg_q}; label acc {msg_l}")
    assert ok_q, msg_q
    assert ok_l, msg_l


def _rank_main(problem, uids_hex, nranks, rank, out, mode, epochs):
    import torch

    torch.cuda.set_device(rank)
    p = np.load(problem)
    uids = [bytes.fromhex(h) for h in uids_hex.split(",")]
    shard = (uids[0], nranks, rank)
    if mode == 1:  # per-epoch errors against the oracle
        np.save(out, jacobi_epoch_errors(p["idx"], p["dist"], shard))
    else:  # one run per seed; each needs its own communicator id, made here from the shared one
        ys = []
        for i, seed in enumerate(SEEDS):
            ys.append(run_session(p["idx"], p["dist"], shard=(uids[i], nranks, rank), mode=mode, epochs=epochs,
                                  seed=seed))
        np.save(out, np.stack(ys))


if __name__ == "__main__":
    _rank_main(sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4]), sys.argv[5], int(sys.argv[6]),
               int(sys.argv[7]))
