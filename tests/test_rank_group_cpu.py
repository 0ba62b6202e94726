"""Rank coordination of the single-process multi-device mode, on the CPU.

fastembedr_b200/csrc/rank_group.h is what the multi-device openTSNE mode
(FASTEMBEDR_B200_DEVICES) routes every collective through.  Here its threads
issue collectives on the tracked stand-in NCCL (tests/fake_nccl.c,
-DFAKE_NCCL_TRACK) while one rank fails mid-run, and the checks are the
properties the mode relies on:

* a rank that fails on the host stops its peers before they enqueue a
  collective it will not join, and no communicator is aborted mid-run;
* a rank whose own enqueue fails after its peers enqueued theirs triggers the
  abort of every communicator, and no NCCL call (collective, second abort or
  destroy) reaches a communicator after its abort;
* on a clean run every rank issues every collective and nothing is aborted.
"""
import os
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    out = tmp_path_factory.mktemp("rank_group") / "rank_group_harness"
    subprocess.run(["g++", "-std=c++17", "-O1", "-pthread", "-DFAKE_NCCL_TRACK", "-x", "c++",
                    os.path.join(HERE, "rank_group_harness.cpp"), "-x", "c",
                    os.path.join(HERE, "fake_nccl.c"), "-o", str(out)], check=True)
    return str(out)


def _run(harness, scenario, nranks, collectives, fail_rank, fail_at, seed):
    res = subprocess.run([harness, scenario, str(nranks), str(collectives), str(fail_rank), str(fail_at),
                          str(seed)], capture_output=True, text=True, timeout=60, check=True)
    fields = dict(item.split("=") for item in res.stdout.split())
    return ([int(v) for v in fields["calls"].split(",")], [int(v) for v in fields["statuses"].split(",")],
            int(fields["aborts"]), int(fields["after_abort"]))


def test_clean_run_issues_everything(harness):
    calls, statuses, aborts, after = _run(harness, "host", 4, 200, -1, -1, 1)
    assert calls == [200] * 4
    assert statuses == [0] * 4
    assert aborts == 0 and after == 0


@pytest.mark.parametrize("seed", range(8))
@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_host_failure_stops_peers_before_their_next_collective(harness, nranks, seed):
    fail_rank = seed % nranks
    fail_at = 5 + 7 * seed
    calls, statuses, aborts, after = _run(harness, "host", nranks, 200, fail_rank, fail_at, seed)
    # Every rank issued exactly the collectives before the failure point: none
    # enqueued the collective the failed rank never joined.
    assert calls == [fail_at] * nranks
    assert statuses[fail_rank] == -1
    assert all(st == 1 for r, st in enumerate(statuses) if r != fail_rank)  # kPeerFailed
    # Nothing was in flight without a peer, so no abort happened mid-run; the
    # tear-down aborts each communicator once, and never after an abort.
    assert aborts == nranks
    assert after == 0


@pytest.mark.parametrize("seed", range(8))
@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_enqueue_failure_aborts_and_no_call_follows(harness, nranks, seed):
    fail_rank = (seed + 1) % nranks
    fail_at = 3 + 11 * seed
    calls, statuses, aborts, after = _run(harness, "enqueue", nranks, 200, fail_rank, fail_at, seed)
    # The failing rank's call fail_at failed.  Its peers had arrived at that
    # collective: each either enqueued it before the abort or found its
    # communicator already aborted (kAborted) and enqueued nothing; none
    # issued one more.
    assert calls[fail_rank] == fail_at
    assert statuses[fail_rank] == 3  # kIssueFailed
    for r in range(nranks):
        if r == fail_rank:
            continue
        assert calls[r] in (fail_at, fail_at + 1)
        assert statuses[r] == (1 if calls[r] == fail_at + 1 else 2)  # kPeerFailed / kAborted
    assert aborts == nranks  # each communicator exactly once
    assert after == 0
