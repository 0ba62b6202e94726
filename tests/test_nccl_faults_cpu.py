"""NCCL failures reach the caller as status 1 with NCCL's message (CPU only).

The library opens NCCL at run time (FASTEMBEDR_B200_NCCL_LIB overrides the
path), so a failing NCCL can be injected on the host: a stand-in library built
here from tests/fake_nccl.c returns error codes from every call, or lacks an
entry point, or the path does not exist.  Each case runs in a fresh process,
because the library resolves NCCL once per process.  No GPU is involved:
fe_b200_nccl_unique_id is the one NCCL entry point that needs no device.
"""
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
    return {"failing": _build(d, "failing"), "incomplete": _build(d, "incomplete", "-DFAKE_NCCL_MISSING_ALLGATHER")}


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
