"""Sharded t-SNE on B200s, one process per GPU, through the C ABI.

Each rank spreads, attracts and updates its own block of points; the charge
grid is summed with an NCCL all-reduce and the updated points are all-gathered
every iteration.  Charges are 64-bit fixed point and every rank reduces the
layout statistics of the gathered layout in one fixed order, so a run on any
number of ranks must give the same bits as a one-rank sharded run; a one-rank
sharded run must give the unsharded session's gradient exactly and its layout
to within the rounding of the (differently ordered) layout-mean sums.

The two-rank test needs two GPUs and is skipped on a one-GPU box.
"""
import os
import subprocess
import sys

if __name__ == "__main__":  # a rank process of the two-GPU test
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import numpy as np
import pytest

from fastembedr_b200 import api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu

N, K, PERPLEXITY = 6000, 45, 15.0  # n >= 4096: the run crosses spatial reorders
EARLY, LATE = 100, 60


def _problem_arrays():
    x, _ = S.gaussian_mixture(S.MixtureSpec(n=N, components=8, seed=3))
    idx, dist = S.exact_knn(x, K)
    return idx, dist, S.tsne_init(N, seed=1)


def run_session(idx, dist, init, shard=None, comm=None):
    """Gradient at the init, then EARLY + LATE iterations: final layout and state."""
    lr_e, lr_l = float(np.float32(N / 12.0)), float(np.float32(N / 1.0))
    with api.TsneSession.from_knn(idx, dist, perplexity=PERPLEXITY, init=init) as s:
        if shard is not None:
            s.shard(*shard)
        if comm is not None:
            s.shard_comm(comm)
        grad, z = s.gradient(12.0)
        s.iterate(EARLY, 12.0, 0.8, lr_e)
        s.iterate(LATE, 1.0, 0.8, lr_l)
        y = s.layout()
        upd, gains = s.state()
    return {"grad": grad, "z": np.float64(z), "y": y, "update": upd, "gains": gains}


@pytest.fixture(scope="module")
def problem(tmp_path_factory):
    idx, dist, init = _problem_arrays()
    path = tmp_path_factory.mktemp("shard") / "problem.npz"
    np.savez(path, idx=idx, dist=dist, init=init)
    return str(path)


def test_one_rank_shard_matches_unsharded(problem):
    p = np.load(problem)
    plain = run_session(p["idx"], p["dist"], p["init"])
    one = run_session(p["idx"], p["dist"], p["init"], shard=(api.nccl_unique_id(), 1, 0))
    assert np.array_equal(one["grad"], plain["grad"])
    assert one["z"] == plain["z"]
    assert np.isfinite(one["y"]).all()
    rel = np.linalg.norm(one["y"] - plain["y"]) / np.linalg.norm(plain["y"])
    assert rel < 1e-3, rel


def test_lent_communicator_serves_sessions_in_turn(problem):
    p = np.load(problem)
    own = run_session(p["idx"], p["dist"], p["init"], shard=(api.nccl_unique_id(), 1, 0))
    with api.NcclComm(api.nccl_unique_id(), 1, 0) as comm:
        for _ in range(2):  # the session closes, the communicator stays usable
            lent = run_session(p["idx"], p["dist"], p["init"], comm=comm)
            for key in ("grad", "z", "y", "update", "gains"):
                assert np.array_equal(lent[key], own[key]), key


def test_shard_rejects_bad_ranks(problem):
    p = np.load(problem)
    with api.TsneSession.from_knn(p["idx"], p["dist"], perplexity=PERPLEXITY, init=p["init"]) as s:
        with pytest.raises(api.CudaBackendError, match="nranks"):
            s.shard(api.nccl_unique_id(), 2, 2)
        with pytest.raises(api.CudaBackendError, match="nranks"):
            s.shard(api.nccl_unique_id(), 0, 0)


JOIN_PROBE = r"""
import sys
sys.path.insert(0, {root!r})
import numpy as np
from fastembedr_b200 import api
try:
    api.NcclComm(api.nccl_unique_id(), 2, 0)  # rank 1 is never started
except api.CudaBackendError as e:
    print("ERROR:", e)
else:
    print("JOINED")
x = np.random.default_rng(0).normal(size=(600, 10)).astype(np.float32)
d = ((x[:, None] - x[None]) ** 2).sum(-1)
np.fill_diagonal(d, np.inf)
idx = np.argsort(d, 1)[:, :20].astype(np.int32)
dist = np.sqrt(np.take_along_axis(d, idx, 1)).astype(np.float32)
with api.NcclComm(api.nccl_unique_id(), 1, 0) as comm:  # the same bounded join, one rank
    with api.TsneSession.from_knn(idx, dist, perplexity=10.0) as s:
        s.shard_comm(comm)
        s.iterate(5, 12.0, 0.8, 50.0)
        print("AFTER", bool(np.isfinite(s.layout()).all()))
"""


def test_peer_that_never_joins_times_out():
    """A rank whose peer never starts gives up after the join limit, aborts the
    communicator and returns status 1; the process and its device stay usable.
    Host side only: no kernel or collective is in flight while it waits."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, FASTEMBEDR_B200_NCCL_INIT_TIMEOUT_S="3", NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", JOIN_PROBE.format(root=root)], env=env, capture_output=True,
                       text=True, timeout=180)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.strip().splitlines()  # NCCL may print its version banner first
    errors = [ln for ln in lines if ln.startswith("ERROR:")]
    assert len(errors) == 1 and "timed out after 3 s" in errors[0] and "aborted" in errors[0], lines
    assert "JOINED" not in lines and lines[-1] == "AFTER True", lines


def _gpu_count():
    import torch

    return torch.cuda.device_count()


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_two_ranks_bit_identical_to_one_rank(problem, tmp_path):
    uid = api.nccl_unique_id()
    procs = []
    for rank in range(2):
        out = tmp_path / f"rank{rank}.npz"
        env = dict(os.environ, NCCL_NVLS_ENABLE="0")
        procs.append((out, subprocess.Popen([sys.executable, __file__, problem, uid.hex(), "2", str(rank), str(out)],
                                            env=env)))
    try:
        codes = [p.wait(timeout=300) for _, p in procs]
    finally:
        for _, p in procs:  # a rank left waiting for a failed peer is ended here
            if p.poll() is None:
                p.kill()
                p.wait()
    assert codes == [0, 0], codes
    p = np.load(problem)
    one = run_session(p["idx"], p["dist"], p["init"], shard=(api.nccl_unique_id(), 1, 0))
    for out, _ in procs:
        got = np.load(out)
        for key in ("grad", "z", "y", "update", "gains"):
            assert np.array_equal(got[key], one[key]), key


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_single_process_two_devices_match_one_rank(problem, tmp_path):
    """FASTEMBEDR_B200_DEVICES=0,1: the unchanged one-shot entry point runs one
    sharded session per device in this process; the layout must be the bits
    of a one-rank sharded session (the decomposition does not change them)."""
    p = np.load(problem)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", FASTEMBEDR_B200_DEVICES="0,1")
    script = (
        "import sys, numpy as np\n"
        f"sys.path.insert(0, {os.path.dirname(os.path.dirname(os.path.abspath(__file__)))!r})\n"
        "from fastembedr_b200 import api\n"
        f"p = np.load({problem!r})\n"
        f"res = api.opentsne_knn(p['idx'], p['dist'], perplexity={PERPLEXITY}, init=p['init'],\n"
        f"                       early_exaggeration_iter={EARLY}, n_iter={LATE})\n"
        f"np.save({str(tmp_path / 'multi.npy')!r}, res.Y)\n")
    r = subprocess.run([sys.executable, "-c", script], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    got = np.load(tmp_path / "multi.npy")
    with api.TsneSession.from_knn(p["idx"], p["dist"], perplexity=PERPLEXITY, init=p["init"]) as s:
        s.shard(api.nccl_unique_id(), 1, 0)
        want = s.run(EARLY, LATE)
    assert np.array_equal(got, want)


INJECT_PROBE = r"""
import os, sys, numpy as np
sys.path.insert(0, {root!r})
from fastembedr_b200 import api
p = np.load({problem!r})
kw = dict(perplexity={perp}, init=p['init'], early_exaggeration_iter={early}, n_iter={late})
try:
    api.opentsne_knn(p['idx'], p['dist'], **kw)
except api.CudaBackendError as e:
    print("ERROR:", e)
else:
    print("RAN")
del os.environ["FASTEMBEDR_B200_INJECT_HOST_FAILURE"]
res = api.opentsne_knn(p['idx'], p['dist'], **kw)  # the same process runs again
np.save({out!r}, res.Y)
print("AFTER")
"""


@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_single_process_host_failure_stops_every_rank(problem, tmp_path):
    """FASTEMBEDR_B200_DEVICES=0,1 with rank 1 failing on the host before its
    41st collective (mid-run, none of its collectives in flight): rank 0 learns
    of it on the host before enqueuing that collective, both ranks stop, the
    call returns status 1 naming the cause, and the same process then runs the
    call again to the bits of a one-rank sharded session.  No collective is left
    waiting on a GPU, so no communicator is aborted with work in flight."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = str(tmp_path / "after.npy")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", FASTEMBEDR_B200_DEVICES="0,1",
               FASTEMBEDR_B200_INJECT_HOST_FAILURE="1:40", FASTEMBEDR_B200_COLLECTIVE_TIMEOUT_S="60")
    script = INJECT_PROBE.format(root=root, problem=problem, perp=PERPLEXITY, early=EARLY, late=LATE, out=out)
    r = subprocess.run([sys.executable, "-c", script], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith(("ERROR:", "RAN", "AFTER"))]
    assert len(lines) == 2 and lines[0].startswith("ERROR:") and lines[1] == "AFTER", r.stdout[-2000:]
    assert "injected host failure of rank 1 before collective 40" in lines[0], lines[0]
    p = np.load(problem)
    with api.TsneSession.from_knn(p["idx"], p["dist"], perplexity=PERPLEXITY, init=p["init"]) as s:
        s.shard(api.nccl_unique_id(), 1, 0)
        want = s.run(EARLY, LATE)
    assert np.array_equal(np.load(out), want)


def _rank_main(problem, uid_hex, nranks, rank, out):
    import torch

    torch.cuda.set_device(rank)
    p = np.load(problem)
    res = run_session(p["idx"], p["dist"], p["init"], shard=(bytes.fromhex(uid_hex), nranks, rank))
    np.savez(out, **res)


if __name__ == "__main__":
    _rank_main(sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4]), sys.argv[5])
