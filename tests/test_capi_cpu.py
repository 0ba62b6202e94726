"""CPU-only checks of the drop-in boundary and the host logic (no GPU needed).

* the C-ABI library loads and exports every function include/fastembedr_b200.h
  declares (which includes every symbol the reference wrapper links against);
* calls that fail before touching a device return status 1 with the
  reference's messages;
* the host-side parameter policies match the reference.
"""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import oracle as O
from fastembedr_b200 import _lib, api
from fastembedr_b200.api import _ptr

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REFERENCE_WRAPPER_SYMBOLS = [
    # every prototype of the extern "C" block in src/embedding_cuda_impl.cpp:24-380
    "fastembedr_cuda_available", "fastembedr_cuda_embedding_last_error", "fastembedr_cuda_embed",
    "fastembedr_cuda_embed_from_knn", "fastembedr_cuda_spectral_init_from_knn",
    "fastembedr_cuda_exact_tsne_from_knn", "fastembedr_cuda_opentsne_fft_from_knn",
    "fastembedr_cuda_opentsne_fft_from_knn_float", "fastembedr_cuda_opentsne_fft_from_device_knn_float",
    "fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_double",
    "fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_float",
    "fastembedr_cuda_umap_from_knn_spectral", "fastembedr_cuda_umap_from_knn_spectral_float",
    "fastembedr_cuda_umap_from_device_knn_spectral_float", "fastembedr_cuda_umap_graph_dump_from_knn",
    "fastembedr_cuda_umap_optimize_coo", "fastembedr_cuda_landmark_tsne_from_device_knn",
    "fastembedr_cuda_landmark_umap_from_device_knn", "fastembedr_cuda_standardize_matrix",
    "fastembedr_cuda_project_embedding", "fastembedr_cuda_interpolate_landmark_layout",
    "fastembedr_cuda_landmark_project_interpolate_knn_confidence", "fastembedr_cuda_knn_structure_score",
    "fastembedr_cuda_silhouette_score", "fastembedr_cuda_matrix_multiply",
    "fastembedr_cuda_raft_tsvd_pca_init",
]


def exported_symbols():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_library_loads_and_exports_header():
    L = _lib.load()
    assert L is not None
    declared = _lib.header_functions()
    assert len(declared) >= 40
    exported = exported_symbols()
    missing = [f for f in declared if f not in exported]
    assert not missing, missing
    for f in declared:
        assert hasattr(L, f)


def test_header_covers_reference_wrapper():
    declared = set(_lib.header_functions())
    assert set(REFERENCE_WRAPPER_SYMBOLS) <= declared


def test_only_the_c_abi_is_exported():
    exported = exported_symbols()
    ours = {s for s in exported if re.match(r"^(fastembedr_cuda_|fe_b200_)", s)}
    assert ours == set(_lib.header_functions())
    assert not any("fe6" in s or "TsneSession" in s for s in exported)


def test_version_string():
    assert "sm_100a" in api.version()


def test_available_false_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert api.cuda_available() is False


@pytest.mark.parametrize("name,nargs", [
    ("fastembedr_cuda_embed", 14), ("fastembedr_cuda_exact_tsne_from_knn", 16),
    ("fastembedr_cuda_standardize_matrix", 6), ("fastembedr_cuda_silhouette_score", 6),
    ("fastembedr_cuda_matrix_multiply", 7), ("fastembedr_cuda_raft_tsvd_pca_init", 5),
])
def test_out_of_scope_symbols_fail_cleanly(name, nargs):
    fn = getattr(_lib.load(), name)
    fn.restype = ctypes.c_int
    args = [ctypes.c_void_p(0)] * nargs
    assert fn(*args) == 1
    assert "not provided by the B200 backend" in _lib.last_error()


def test_pca_init_variants_validate_before_device_work():
    """The PCA-initialised entry points compute their start on the device
    (no RAFT needed); a missing data matrix or too few features is rejected
    before any device call."""
    L = _lib.load()
    out = np.zeros((10, 2), np.float32)
    fout = out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    idx = np.zeros(30, np.int32)
    dist = np.ones(30, np.float32)
    x = np.zeros(10, np.float64)
    for fn in (L.fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_double,
               L.fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_float):
        args = [ctypes.c_void_p(idx.ctypes.data), ctypes.c_void_p(dist.ctypes.data), None, 2, 10, 3, 2, 1.0, 10, 10,
                12.0, 1.0, 0.0, 1, 0.8, 0.8, 0.01, 5.0, 1, 0, fout]
        assert fn(*args) == 1
        assert "PCA" in _lib.last_error()
        args[2] = ctypes.c_void_p(x.ctypes.data)
        args[3] = 1  # one feature
        assert fn(*args) == 1
        assert _lib.last_error() == "invalid dimensions in device PCA initialization"


def test_parameter_validation_precedes_device_work():
    L = _lib.load()
    out = np.zeros((10, 2), np.float32)
    fout = out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    idx = np.zeros(30, np.int32)
    dist = np.ones(30, np.float32)
    base = [ctypes.c_void_p(idx.ctypes.data), ctypes.c_void_p(dist.ctypes.data), None, 0, 10, 3, 2, 1.0,
            10, 10, 12.0, 1.0, 0.0, 1, 0.8, 0.8, 0.01, 5.0, 1, 0, fout]
    cases = {4: 1, 5: 300, 6: 3, 7: 0.0, 8: -1, 10: 0.0, 16: 0.0}
    for pos, bad in cases.items():
        args = list(base)
        args[pos] = bad
        assert L.fastembedr_cuda_opentsne_fft_from_knn_float(*args) == 1
        assert _lib.last_error() == "invalid CUDA openTSNE FFT-grid dimensions or parameters"
    args = list(base)
    args[0] = None
    assert L.fastembedr_cuda_opentsne_fft_from_knn_float(*args) == 1
    assert _lib.last_error() == "null CUDA openTSNE input pointer"
    args = list(base)
    args[3] = 1  # has_init without init
    assert L.fastembedr_cuda_opentsne_fft_from_knn_float(*args) == 1


def test_umap_validation_precedes_device_work():
    with pytest.raises(api.CudaBackendError, match="invalid CUDA COO UMAP optimization parameters"):
        api.umap_optimize_coo([0], [1], [1.0], [1.0], np.zeros((2, 2), np.float32), n_epochs=0)
    with pytest.raises(api.CudaBackendError, match="invalid CUDA COO UMAP optimization parameters"):
        api.umap_optimize_coo([0], [1], [1.0], [1.0], np.zeros((2, 2), np.float32), learning_rate=0.0)
    with pytest.raises(ValueError):
        api.umap_optimize_coo([0, 1], [1], [1.0], [1.0], np.zeros((2, 2), np.float32))


def test_fused_umap_validation_precedes_device_work():
    """The reference's checks and messages (src/embedding_cuda_kernels.cpp:4984-4992,
    5217-5224, 4817-4825), before any CUDA call."""
    L = _lib.load()
    idx = np.zeros(40, np.int32)
    dist = np.ones(40, np.float32)
    out = np.zeros((10, 2), np.float32)
    fout = out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    base = [ctypes.c_void_p(idx.ctypes.data), ctypes.c_void_p(dist.ctypes.data), 10, 4, 20, 5, 1.0, 1.5, 0.9, 1.0,
            30, 42, 0, 0, fout]
    for pos, bad, msg in ((3, 300, "invalid host CUDA UMAP dimensions"), (2, 1, "invalid host CUDA UMAP dimensions"),
                          (4, 0, "invalid fused CUDA UMAP dimensions or parameters"),
                          (6, 0.0, "invalid fused CUDA UMAP dimensions or parameters"),
                          (10, 0, "invalid fused CUDA UMAP dimensions or parameters"),
                          (0, None, "null host pointer")):
        args = list(base)
        args[pos] = bad
        assert L.fastembedr_cuda_umap_from_knn_spectral_float(*args) == 1
        assert _lib.last_error() == msg
    dev = base[:14] + [0, fout]
    dev[0] = None
    assert L.fastembedr_cuda_umap_from_device_knn_spectral_float(*dev) == 1
    assert _lib.last_error() == "null device pointer"
    i_out = np.zeros(400, np.int32)
    f_out = np.zeros(400, np.float32)
    w_out, c_out = ctypes.c_int(0), ctypes.c_int(0)
    ip = i_out.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
    fp = f_out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    assert L.fastembedr_cuda_umap_graph_dump_from_knn(
        ctypes.c_void_p(idx.ctypes.data), ctypes.c_void_p(dist.ctypes.data), 10, 0, 0, ip, ip, fp, fp,
        ctypes.byref(w_out), ctypes.byref(c_out)) == 1
    assert _lib.last_error() == "invalid CUDA UMAP graph dump dimensions"


def test_umap_config_size_rules():
    assert api.umap_config(20000, 15)["n_epochs"] == 200 and api.umap_config(20000, 15)["spectral_n_iter"] == 30
    assert api.umap_config(20000, 30)["spectral_n_iter"] == 20
    assert api.umap_config(1000, 15)["n_epochs"] == 500 and api.umap_config(1000, 15)["spectral_n_iter"] == 60
    assert api.umap_config(100, 15)["spectral_n_iter"] == 50


def test_tsne_auto_parameters_policy():
    # Values asserted by the reference's own tests (tests/testthat/test-tsne.R:31-56).
    p = api.tsne_auto_parameters(150, 30, None)
    assert p["perplexity"] == 10 and p["learning_rate"] == 150 / p["early_exaggeration"]
    assert api.tsne_auto_parameters(70000, 90, None)["perplexity"] == 30
    assert api.tsne_auto_parameters(10000, 90, 30.0)["learning_rate"] == pytest.approx(10000 / 12)


@pytest.mark.skipif(not O.ref_available(), reason="compiled reference not present")
@pytest.mark.parametrize("n,k,perp,missing", [(150, 30, 0.0, True), (70000, 90, 0.0, True),
                                              (1000, 45, 15.0, False), (50, 200, 80.0, False)])
def test_tsne_auto_parameters_against_reference(n, k, perp, missing):
    ref = O.ref_tsne_auto_parameters(n, k, perp, missing)
    ours = api.tsne_auto_parameters(n, k, None if missing else perp)
    for key in ("perplexity", "n_neighbors", "early_exaggeration", "learning_rate",
                "early_exaggeration_iter", "n_iter"):
        assert ours[key] == pytest.approx(ref[key]), key


def test_find_ab_params_matches_reference(umap_scalar_golden):
    g = umap_scalar_golden
    for md, (a, b) in zip(g["ab_min_dist"], g["ab"]):
        ra, rb = api.find_ab_params(1.0, float(md))
        assert ra == pytest.approx(a, rel=1e-12) and rb == pytest.approx(b, rel=1e-12)


def test_index_offset_detection():
    assert api.resolve_index_offset(np.array([[1, 2], [2, 1]])) == 1
    assert api.resolve_index_offset(np.array([[0, 1], [1, 0]])) == 0
    assert api.resolve_index_offset(np.array([[1, 3], [2, 1]])) == 0  # 3 > n


def test_synthetic_configs_shapes():
    from fastembedr_b200 import synthetic as S

    x, lab = S.gaussian_mixture(S.MixtureSpec(n=500, components=5, dirichlet_weights=True, anisotropic=True))
    assert x.shape == (500, 50) and x.dtype == np.float32 and lab.max() < 5
    idx, dist = S.exact_knn(x, 10)
    assert idx.shape == (500, 10) and (idx != np.arange(500)[:, None]).all()
    assert (np.diff(dist, axis=1) >= 0).all()
    d = np.linalg.norm(x[:, None, :].astype(np.float64) - x[None, :, :], axis=-1)
    np.fill_diagonal(d, np.inf)
    np.testing.assert_allclose(np.sort(d, axis=1)[:, :10], dist, rtol=1e-5)


def test_extension_entry_points_validate_before_device_work():
    """The library's own entry points (sessions, epoch ranges, no-allocation
    epochs, NCCL id and communicator) reject bad arguments with status 1 and a
    message before any CUDA or NCCL call."""
    L = _lib.load()
    h = ctypes.c_void_p()
    idx = np.zeros((10, 3), np.int32)
    dist = np.ones((10, 3), np.float32)
    ip, dp = ctypes.c_void_p(idx.ctypes.data), ctypes.c_void_p(dist.ctypes.data)

    def rejects(rc, msg):
        assert rc == 1
        assert msg in _lib.last_error(), _lib.last_error()

    # t-SNE sessions
    rejects(L.fe_b200_tsne_create(None, dp, 10, 3, 0, 5.0, None, 1, 0, 0, ctypes.byref(h)),
            "null CUDA openTSNE input pointer")
    for n, k, perp in ((1, 3, 5.0), (10, 0, 5.0), (10, 300, 5.0), (10, 3, 0.0)):
        rejects(L.fe_b200_tsne_create(ip, dp, n, k, 0, perp, None, 1, 0, 0, ctypes.byref(h)),
                "invalid CUDA openTSNE FFT-grid dimensions or parameters")
    rp = np.array([0, 1, 2], np.int32)
    col = np.array([1, 0], np.int32)
    val = np.full(2, 0.5, np.float32)
    y = np.zeros((2, 2), np.float32)
    rejects(L.fe_b200_tsne_create_csr(_ptr(rp, ctypes.c_int), _ptr(col, ctypes.c_int), _ptr(val, ctypes.c_float), 1,
                                      _ptr(y, ctypes.c_float), 0, ctypes.byref(h)), "invalid CSR session arguments")
    rejects(L.fe_b200_tsne_iterate(None, 1, 1.0, 0.8, 1.0, 0.01, 5.0), "invalid t-SNE session call")
    # UMAP sessions and epoch ranges
    rejects(L.fe_b200_umap_create(None, dp, 10, 3, 0, 0, 0, 30, 1, ctypes.byref(h)), "null pointer")
    rejects(L.fe_b200_umap_create(ip, dp, 1, 3, 0, 0, 0, 30, 1, ctypes.byref(h)),
            "invalid UMAP session dimensions or parameters")
    heads = np.array([0, 1], np.int32)
    tails = np.array([1, 0], np.int32)
    eps = np.ones(2, np.float32)
    lay = np.zeros((2, 2), np.float32)
    args = [_ptr(heads, ctypes.c_int), _ptr(tails, ctypes.c_int), _ptr(eps, ctypes.c_float), 2,
            _ptr(lay, ctypes.c_float), 2]
    tail = [5, 1.0, 1.5769434601962196, 0.8950608781227859, 1.0, 42, 0, 0, None]
    for b, e in ((-1, 2), (3, 2), (0, 11)):
        rejects(L.fe_b200_umap_epochs(*args, b, e, 10, *tail), "invalid epoch range")
    # no-allocation epochs: the vertex cap and the range
    na = [ctypes.c_void_p(1), ctypes.c_void_p(1), ctypes.c_void_p(1), 2, ctypes.c_void_p(1)]
    rejects(L.fe_b200_umap_epochs_noalloc(*na, 2_000_000, 0, 1, 10, 5, 1.0, 1.5, 0.9, 1.0, 42, 1, None),
            "exceeds the fixed scratch capacity")
    rejects(L.fe_b200_umap_epochs_noalloc(*na, 2, 5, 1, 10, 5, 1.0, 1.5, 0.9, 1.0, 42, 1, None),
            "invalid epoch range")
    rejects(L.fe_b200_umap_epochs_noalloc(None, *na[1:], 2, 0, 1, 10, 5, 1.0, 1.5, 0.9, 1.0, 42, 1, None),
            "null device pointer")
    # NCCL id and communicator
    small = (ctypes.c_ubyte * 16)()
    rejects(L.fe_b200_nccl_unique_id(small, 16), "at least 128 bytes")
    uid = (ctypes.c_ubyte * 128)()
    rejects(L.fe_b200_comm_create(uid, 16, 2, 0, ctypes.byref(h)), "invalid communicator call")
    for nranks, rank in ((0, 0), (2, 2), (2, -1)):
        rejects(L.fe_b200_comm_create(uid, 128, nranks, rank, ctypes.byref(h)), "need nranks >= 1")
    rejects(L.fe_b200_tsne_shard_comm(None, None), "invalid t-SNE shard call")
    L.fe_b200_comm_destroy(None)  # a null communicator is ignored


def test_multi_device_list_is_checked_before_device_work(monkeypatch):
    """FASTEMBEDR_B200_DEVICES (one process, several GPUs behind the one-shot
    entry points): a malformed or repeated list is rejected with status 1
    before any device call; a list of two or more devices needs the devices
    (on this GPU-less host the device query itself fails cleanly)."""
    L = _lib.load()
    out = np.zeros((10, 2), np.float32)
    fout = out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    idx = np.zeros(30, np.int32)
    dist = np.ones(30, np.float32)
    args = [ctypes.c_void_p(idx.ctypes.data), ctypes.c_void_p(dist.ctypes.data), None, 0, 10, 3, 2, 1.0,
            10, 10, 12.0, 1.0, 0.0, 1, 0.8, 0.8, 0.01, 5.0, 1, 0, fout]
    for value, msg in (("x", "is not a device ordinal"), ("0,", "is not a device ordinal"),
                       ("1,1", "lists device 1 twice"), ("0,1", "cudaGetDeviceCount(FASTEMBEDR_B200_DEVICES)")):
        monkeypatch.setenv("FASTEMBEDR_B200_DEVICES", value)
        assert L.fastembedr_cuda_opentsne_fft_from_knn_float(*args) == 1
        assert msg in _lib.last_error(), (value, _lib.last_error())
    monkeypatch.setenv("FASTEMBEDR_B200_DEVICES", "0")  # one device: the ordinary path
    assert L.fastembedr_cuda_opentsne_fft_from_knn_float(*args) == 1
    assert "FASTEMBEDR_B200_DEVICES" not in _lib.last_error()


def _reference_prototype_block():
    """The reference wrapper's own extern "C" prototype block
    (src/embedding_cuda_impl.cpp:24-380), read from the reference sources at
    test time; None where they are absent."""
    src = os.environ.get("FASTEMBEDR_REFERENCE_SRC") or os.path.join(os.path.dirname(ROOT), "reference", "src")
    path = os.path.join(src, "embedding_cuda_impl.cpp")
    if not os.path.exists(path):
        return None
    lines = open(path).read().splitlines()
    start = lines.index('extern "C" {')
    end = lines.index("}", start)
    return "\n".join(lines[start:end + 1]) + "\n"


def _compile_against(header_text, block, tmp_path):
    inc = tmp_path / "inc"
    inc.mkdir(exist_ok=True)
    (inc / "fastembedr_b200.h").write_text(header_text)
    tu = tmp_path / "boundary.cpp"
    # R's opaque object handle, for the two helpers the wrapper declares in
    # the block and defines itself (src/embedding_cuda_impl.cpp:230-231).
    tu.write_text('#include "fastembedr_b200.h"\ntypedef struct SEXPREC* SEXP;\n' + block)
    return subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", str(inc), str(tu)],
                          capture_output=True, text=True)


def test_header_compiles_against_reference_prototypes(tmp_path):
    """Every prototype the reference wrapper declares for the backend library,
    compiled in one translation unit with include/fastembedr_b200.h: a C-linkage
    function declared twice with different parameter or return types does not
    compile, so the signatures agree type for type, not only by name.  A copy
    of the header with one argument type changed must then fail."""
    block = _reference_prototype_block()
    if block is None:
        pytest.skip("reference sources not present on this host")
    header = open(os.path.join(ROOT, "include", "fastembedr_b200.h")).read()
    ok = _compile_against(header, block, tmp_path)
    assert ok.returncode == 0, ok.stderr[-3000:]
    # Negative control: the last argument kind of the UMAP COO optimizer.
    bad = header.replace("int optimizer_mode, float* out);", "float optimizer_mode, float* out);", 1)
    assert bad != header
    broken = _compile_against(bad, block, tmp_path)
    assert broken.returncode != 0
    assert "fastembedr_cuda_umap_optimize_coo" in broken.stderr
