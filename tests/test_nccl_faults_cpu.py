"""NCCL failures reach the caller as status 1 with NCCL's message (CPU only).

The library opens NCCL at run time (FASTEMBEDR_B200_NCCL_LIB overrides the
path), so a failing NCCL can be injected on the host: a stand-in library built
here from tests/fake_nccl.c returns error codes from every call, or lacks an
entry point, or the path does not exist, or models the join of a communicator
whose peers take a number of polls to arrive or never arrive.  Each case runs
in a fresh process, because the library resolves NCCL once per process.  No GPU
is involved: fe_b200_nccl_unique_id and fe_b200_comm_create reach NCCL before
any device call, and the stand-in touches no device.
"""
import time
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

PROBE = r"""
import sys
sys.path.insert(0, {root!r})
from fastembedr_b200 import api
try:
    api.nccl_unique_id()
except api.CudaBackendError as e:
    print("ERROR:", e)
else:
    print("OK")
"""


JOIN_PROBE = r"""
import ctypes, sys, time
sys.path.insert(0, {root!r})
from fastembedr_b200 import api
t0 = time.perf_counter()
try:
    comm = api.NcclComm(bytes(128), 2, 0)
except api.CudaBackendError as e:
    out = "ERROR: " + str(e)
else:
    out = "OK"
    comm.close()
secs = time.perf_counter() - t0
fake = ctypes.CDLL({fake!r})
print(out)
print("COUNTS", fake.fake_nccl_aborts(), fake.fake_nccl_polls(), fake.fake_nccl_last_blocking(), secs)
"""


def _build(tmp_path, name, *flags):
    out = tmp_path / f"{name}.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", *flags, "-o", str(out), os.path.join(HERE, "fake_nccl.c")],
                   check=True)
    return str(out)


def _probe(nccl_path):
    env = dict(os.environ, FASTEMBEDR_B200_NCCL_LIB=nccl_path)
    r = subprocess.run([sys.executable, "-c", PROBE.format(root=ROOT)], env=env, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    return r.stdout.strip().splitlines()[-1]


@pytest.fixture(scope="module")
def fakes(tmp_path_factory):
    d = tmp_path_factory.mktemp("fake_nccl")
    return {"failing": _build(d, "failing"), "incomplete": _build(d, "incomplete", "-DFAKE_NCCL_MISSING_ALLGATHER"),
            "never_joins": _build(d, "never_joins", "-DFAKE_NCCL_JOIN_POLLS=-1"),
            "slow_join": _build(d, "slow_join", "-DFAKE_NCCL_JOIN_POLLS=50")}


def _join(nccl_path, limit_s=None):
    """Makes a 2-rank communicator as rank 0 through the stand-in: the probe's
    outcome line and (aborts, polls, config.blocking seen, seconds)."""
    env = dict(os.environ, FASTEMBEDR_B200_NCCL_LIB=nccl_path)
    env.pop("FASTEMBEDR_B200_NCCL_INIT_TIMEOUT_S", None)
    if limit_s is not None:
        env["FASTEMBEDR_B200_NCCL_INIT_TIMEOUT_S"] = str(limit_s)
    r = subprocess.run([sys.executable, "-c", JOIN_PROBE.format(root=ROOT, fake=nccl_path)], env=env,
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.strip().splitlines()
    counts = lines[-1].split()
    return lines[-2], (int(counts[1]), int(counts[2]), int(counts[3]), float(counts[4]))


def test_nccl_error_code_becomes_status_1_with_its_message(fakes):
    out = _probe(fakes["failing"])
    assert out.startswith("ERROR:"), out
    assert "ncclGetUniqueId" in out and "no usable network interface" in out and "code 2" in out


def test_missing_nccl_symbol_is_reported(fakes):
    out = _probe(fakes["incomplete"])
    assert "NCCL symbol ncclAllGather not found" in out, out


def test_missing_nccl_library_is_reported(tmp_path):
    out = _probe(str(tmp_path / "no_such_libnccl.so"))
    assert "cannot load NCCL" in out, out


def test_real_nccl_still_works_without_the_override():
    env = {k: v for k, v in os.environ.items() if k != "FASTEMBEDR_B200_NCCL_LIB"}
    r = subprocess.run([sys.executable, "-c", PROBE.format(root=ROOT)], env=env, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip().splitlines()[-1] == "OK"


def test_peer_that_never_joins_times_out_and_aborts(fakes):
    out, (aborts, polls, blocking, secs) = _join(fakes["never_joins"], limit_s=0.5)
    assert out.startswith("ERROR:"), out
    assert "timed out after 0.5 s" in out and "1 rank(s) to join" in out and "aborted" in out, out
    assert aborts == 1  # NCCL's join threads are ended, not left waiting
    assert blocking == 0  # the bounded join makes the communicator nonblocking
    assert polls > 10 and 0.5 <= secs < 30, (polls, secs)


def test_slow_join_within_the_limit_succeeds(fakes):
    out, (aborts, polls, blocking, _) = _join(fakes["slow_join"], limit_s=30)
    assert out == "OK", out
    assert (aborts, polls, blocking) == (0, 51, 0)


def test_without_a_limit_the_join_is_the_blocking_call(fakes):
    out, (aborts, polls, blocking, _) = _join(fakes["slow_join"])
    assert out == "OK", out
    assert (aborts, polls, blocking) == (0, 0, -1)  # ncclCommInitRank, no config, no polling


def test_bounded_join_reports_nccl_errors(fakes):
    out, (aborts, _, blocking, _) = _join(fakes["failing"], limit_s=5)
    assert "ncclCommInitRankConfig" in out and "remote process exited" in out and "code 6" in out, out
    assert blocking == 0 and aborts == 0  # no communicator came back, nothing to abort
