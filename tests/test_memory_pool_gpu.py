"""Device memory retained between calls (a stream-ordered pool per GPU).

A call's device buffers come from a pool that keeps freed blocks mapped for the
next call (up to FASTEMBEDR_B200_RETAIN_MB); fe_b200_release_memory hands them
back to the driver.  Results must not depend on where the buffers come from:
a call with retention off (plain cudaMalloc / cudaFree, set in a child process
because the variable is read once per process) reproduces the layout bit for
bit.
"""
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

from fastembedr_b200 import api
from fastembedr_b200 import synthetic as S

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KW = dict(perplexity=30.0, early_exaggeration_iter=30, n_iter=30)


@pytest.fixture(scope="module")
def knn_20k():
    x, _ = S.gaussian_mixture(S.CONFIGS["tsne_70k"])
    idx, dist = S.exact_knn(x[:20_000], 90, device="cuda")
    return idx, dist, S.tsne_init(20_000, seed=2)


def test_release_returns_retained_memory(knn_20k):
    import torch

    idx, dist, init = knn_20k
    torch.cuda.init()
    api.release_memory()
    free0 = torch.cuda.mem_get_info()[0]
    api.opentsne_knn(idx, dist, init=init, **KW)
    free1 = torch.cuda.mem_get_info()[0]
    api.release_memory()
    free2 = torch.cuda.mem_get_info()[0]
    print(f"free memory: before {free0 / 2**20:.0f} MiB, after the call {free1 / 2**20:.0f} MiB, "
          f"after release {free2 / 2**20:.0f} MiB")
    assert free1 < free0 - (64 << 20)        # the call's buffers stay mapped
    assert free2 > free1 + (64 << 20)        # and go back on request
    assert abs(free2 - free0) <= (64 << 20)


def test_layout_does_not_depend_on_the_allocator(knn_20k):
    idx, dist, init = knn_20k
    pooled = api.opentsne_knn(idx, dist, init=init, **KW).Y
    code = ("import sys, numpy as np; sys.path.insert(0, '.');"
            "from fastembedr_b200 import api;"
            "d = np.load(sys.argv[1]);"
            "y = api.opentsne_knn(d['idx'], d['dist'], init=d['init'], perplexity=30.0,"
            " early_exaggeration_iter=30, n_iter=30).Y;"
            "np.save(sys.argv[2], y)")
    with tempfile.TemporaryDirectory() as tmp:
        src, out = os.path.join(tmp, "knn.npz"), os.path.join(tmp, "y.npy")
        np.savez(src, idx=idx, dist=dist, init=init)
        env = dict(os.environ, FASTEMBEDR_B200_RETAIN_MB="0")
        r = subprocess.run([sys.executable, "-c", code, src, out], cwd=ROOT, env=env, capture_output=True,
                           text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        plain = np.load(out)
    assert np.array_equal(pooled, plain)


def test_session_closed_with_another_device_current(knn_20k):
    """A session's buffers go back to the pool of the GPU that holds them even
    when the caller has another GPU current when it closes the session (as
    cudaFree would); that GPU's pool then serves a new session."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    idx, dist, init = knn_20k
    with torch.cuda.device(1):
        s = api.TsneSession.from_knn(idx, dist, perplexity=30.0, init=init)
        s.iterate(4, 12.0, 0.8, float(np.float32(idx.shape[0] / 12.0)))
        want = s.layout()
    with torch.cuda.device(0):
        s.close()
    with torch.cuda.device(1):
        with api.TsneSession.from_knn(idx, dist, perplexity=30.0, init=init) as s2:
            s2.iterate(4, 12.0, 0.8, float(np.float32(idx.shape[0] / 12.0)))
            assert np.array_equal(s2.layout(), want)
        api.release_memory()
